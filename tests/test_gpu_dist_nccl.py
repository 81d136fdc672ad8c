"""Data parallel over NCCL on 2 GPUs against 1 GPU: the same seeded model
trained on the full batch (world 1) and on half batches per rank (world 2,
values-only gradient all-reduce with ReduceOp.AVG, SET update on rank 0 and
topology broadcast).  The global losses agree to rounding (the all-reduce
sums in a different order), and after the router step every rank holds the
same masks.  Skipped with fewer than 2 GPUs."""
import multiprocessing as mp
import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu

STEPS, UPDATE_FREQ, BATCH = 6, 4, 64


def _setup(device):
    import sparsecore_b200 as sl

    torch.manual_seed(0)
    model = torch.nn.Sequential(sl.SparseLinear(96, 64, sparsity=0.8, device=device), torch.nn.ReLU(),
                                sl.SparseLinear(64, 10, sparsity=0.8, device=device))
    algo = sl.SET(sparsity=0.8, drop_fraction=0.3, update_freq=UPDATE_FREQ, seed=5)
    model.apply(algo)
    opt = torch.optim.SGD(model.parameters(), lr=0.1)
    g = torch.Generator().manual_seed(11)
    x = torch.randn(BATCH, 96, generator=g)
    y = torch.randint(0, 10, (BATCH,), generator=g)
    return model, algo, opt, x, y


def _world1():
    dev = torch.device("cuda", 0)
    model, algo, opt, x, y = _setup(dev)
    x, y = x.to(dev), y.to(dev)
    losses = []
    for _ in range(STEPS):
        opt.zero_grad(set_to_none=True)
        loss = torch.nn.functional.cross_entropy(model(x), y)
        loss.backward()
        opt.step()
        algo.step()
        losses.append(float(loss))
    return losses


def _rank(rank, world, port, q, overlap=False):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        torch.cuda.set_device(rank)
        import torch.distributed as dist

        dist.init_process_group("nccl", rank=rank, world_size=world)
        from sparsecore_b200.dist import SparseDataParallel, sync_after_router_step

        dev = torch.device("cuda", rank)
        model, algo, opt, x, y = _setup(dev)
        shard = BATCH // world
        xs, ys = x[rank * shard:(rank + 1) * shard].to(dev), y[rank * shard:(rank + 1) * shard].to(dev)
        if overlap:
            from sparsecore_b200 import ops

            ops.set_async_weight_grad(True)  # packs + bucket all-reduces start during backward
        ddp = SparseDataParallel(model, overlap=overlap, bucket_mb=0.01)
        losses = []
        for _ in range(STEPS):
            opt.zero_grad(set_to_none=True)
            loss = torch.nn.functional.cross_entropy(model(xs), ys)
            loss.backward()
            ddp.allreduce_grads()
            opt.step()
            algo.step()
            sync_after_router_step(ddp, algo)
            g = loss.detach().clone()
            dist.all_reduce(g, op=dist.ReduceOp.AVG)
            losses.append(float(g))
        q.put((rank, losses, ddp.topology_checksum()))
        dist.destroy_process_group()
    except Exception as e:  # report instead of hanging the parent
        q.put((rank, repr(e), None))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("overlap", [False, True])
def test_two_gpu_data_parallel_matches_one_gpu(overlap):
    """overlap=True: per-layer packs and bucketed all-reduces launched from
    the weight-gradient side stream during backward (buckets of ~10 KB here,
    so each layer is its own bucket)."""
    want = _world1()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q, overlap)) for r in range(2)]
    for p in procs:
        p.start()
    out = {}
    for _ in procs:
        rank, losses, checks = q.get(timeout=300)
        out[rank] = (losses, checks)
    for p in procs:
        p.join(timeout=60)
    for r in (0, 1):
        assert isinstance(out[r][0], list), out[r][0]
    # Identical up to the first update (exact masks, rounding-level values) ...
    assert out[0][0][:UPDATE_FREQ] == pytest.approx(want[:UPDATE_FREQ], rel=1e-5, abs=1e-6)
    assert out[0][0] == out[1][0]
    # ... and after the router step both ranks hold rank 0's masks.
    assert out[0][1] == out[1][1] and len(set(out[0][1])) == 1
    assert all(torch.isfinite(torch.tensor(out[0][0])))
