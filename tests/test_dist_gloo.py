"""Data-parallel host logic on world-size-2 gloo ranks (CPU, no GPU).

``SparseDataParallel`` takes the pack / unpack / offsets steps as callables;
here they are CPU stand-ins with the semantics of sl_pack_live /
sl_unpack_live / sl_exclusive_scan (live slots of row i are
[row_start[i], row_start[i] + row_nnz[i]); padding never travels), and the
layers are CPU fakes with the attributes the helper reads.  Covered: the
values-only gradient all-reduce (AVG), the topology broadcast from rank 0,
the mask checksum, and a rank that fails before the collective (the other
rank's collective ends with an error instead of hanging).
"""
import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


class FakeCSR:
    def __init__(self, nrows, ncols, row_nnz, cap_per_row, seed):
        g = torch.Generator().manual_seed(seed)
        self.nrows, self.ncols = nrows, ncols
        self.row_capacity = torch.full((nrows,), cap_per_row, dtype=torch.int32)
        self.row_start = torch.arange(nrows, dtype=torch.int32) * cap_per_row
        self.row_nnz = torch.tensor(row_nnz, dtype=torch.int32)
        self.total_capacity = nrows * cap_per_row
        self.values = torch.zeros(self.total_capacity)
        self.col_indices = torch.full((self.total_capacity,), -1, dtype=torch.int32)
        for i, n in enumerate(row_nnz):
            s = i * cap_per_row
            self.col_indices[s:s + n] = torch.randperm(ncols, generator=g)[:n].sort().values.int()
            self.values[s:s + n] = torch.randn(n, generator=g)
        self.device = torch.device("cpu")
        self.topology_version = 0
        self.topology_version_ = 0
        self._nnz = int(sum(row_nnz))

    @property
    def nnz(self):
        return self._nnz

    def _sync_row_nnz_from_device(self):
        self._nnz = int(self.row_nnz.sum())
        self.topology_version = self.topology_version_


class FakeLayer:
    def __init__(self, csr):
        self._csr = csr
        self._values = torch.nn.Parameter(csr.values)


def cpu_offsets(layer):
    return torch.cumsum(layer._csr.row_nnz, 0, dtype=torch.int32) - layer._csr.row_nnz


def cpu_pack(layer, offsets, src, dst):
    c = layer._csr
    for i in range(c.nrows):
        n, s, o = int(c.row_nnz[i]), int(c.row_start[i]), int(offsets[i])
        dst[o:o + n] = src[s:s + n]


def cpu_unpack(layer, offsets, src, dst):
    c = layer._csr
    for i in range(c.nrows):
        n, s, o = int(c.row_nnz[i]), int(c.row_start[i]), int(offsets[i])
        dst[s:s + n] = src[o:o + n]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port, timeout_s=30):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=timeout_s))


def _make(rank):
    from sparsecore_b200.dist import SparseDataParallel

    layers = [FakeLayer(FakeCSR(4, 10, [3, 0, 5, 2], 6, seed=1)),
              FakeLayer(FakeCSR(3, 7, [1, 4, 2], 5, seed=2))]
    dense = torch.nn.Linear(3, 2)
    model = torch.nn.ModuleList([dense])
    ddp = SparseDataParallel(model, pack=cpu_pack, unpack=cpu_unpack, offsets=cpu_offsets,
                             sparse_layers=layers)
    # rank-dependent gradients: live slots = rank + 1 + slot index, padding = -99
    for L in layers:
        g = torch.full_like(L._values, -99.0)
        c = L._csr
        for i in range(c.nrows):
            s, n = int(c.row_start[i]), int(c.row_nnz[i])
            g[s:s + n] = rank + 1 + torch.arange(n, dtype=torch.float32)
        L._values.grad = g
    for p in dense.parameters():
        p.grad = torch.full_like(p, float(10 * (rank + 1)))
    return ddp, layers, dense


def _worker_allreduce(rank, world, port, q):
    try:
        _init(rank, world, port)
        ddp, layers, dense = _make(rank)
        ddp.allreduce_grads()
        ok = True
        mean_rank = sum(r + 1 for r in range(world)) / world
        for L in layers:
            c, g = L._csr, L._values.grad
            for i in range(c.nrows):
                s, n, cap = int(c.row_start[i]), int(c.row_nnz[i]), int(c.row_capacity[i])
                ok &= torch.allclose(g[s:s + n], mean_rank + torch.arange(n, dtype=torch.float32))
                ok &= bool((g[s + n:s + cap] == -99.0).all())  # padding untouched
        for p in dense.parameters():
            ok &= bool((p.grad == 10 * mean_rank).all())
        # bucket holds live slots + dense only
        ok &= ddp.bucket_numel == sum(L._csr.nnz for L in layers) + 3 * 2 + 2
        q.put((rank, bool(ok)))
    except Exception as e:  # pragma: no cover - reported to the parent
        q.put((rank, repr(e)))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def _worker_broadcast(rank, world, port, q):
    try:
        _init(rank, world, port)
        ddp, layers, _ = _make(rank)
        if rank == 1:  # diverge rank 1's masks and values
            for L in layers:
                L._csr.col_indices.add_(1)
                L._csr.values.mul_(3.0)
                L._csr.row_nnz[0] = 0
        from sparsecore_b200 import ops

        # Both ranks cached a transpose at the same topology version, built
        # from different masks on rank 1: the broadcast must drop it.
        for L in layers:
            ops._transpose_cache[id(L._csr)] = (L._csr.topology_version, (L._csr.nrows, L._csr.ncols),
                                                "stale W^T", "stale perm")
        before = ddp.topology_checksum()
        ddp.broadcast_topology(src=0)
        after = ddp.topology_checksum()
        ref = [FakeCSR(4, 10, [3, 0, 5, 2], 6, seed=1), FakeCSR(3, 7, [1, 4, 2], 5, seed=2)]
        ok = before[0] != before[1] and after[0] == after[1]
        for L, R in zip(layers, ref):
            ok &= torch.equal(L._csr.col_indices, R.col_indices)
            ok &= torch.equal(L._csr.values, R.values)
            ok &= torch.equal(L._csr.row_nnz, R.row_nnz)
            ok &= L._values.data_ptr() == L._csr.values.data_ptr()  # alias kept
            ok &= id(L._csr) not in ops._transpose_cache  # no stale W^T survives
        q.put((rank, bool(ok)))
    except Exception as e:  # pragma: no cover
        q.put((rank, repr(e)))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def _worker_rank_fails(rank, world, port, q):
    _init(rank, world, port, timeout_s=5)
    ddp, _, _ = _make(rank)
    if rank == 1:
        q.put((rank, "left"))
        q.close()
        q.join_thread()  # flush before leaving
        os._exit(0)  # leaves between steps, without joining the collective
    try:
        ddp.allreduce_grads()
        q.put((rank, "no error"))
    except Exception as e:  # the surviving rank learns of it on the host
        q.put((rank, "raised " + type(e).__name__))


def _run(fn, world=2, timeout=90):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=fn, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = {}
    for _ in range(world):
        r, v = q.get(timeout=timeout)
        out[r] = v
    for p in procs:
        p.join(timeout=timeout)
        if p.is_alive():
            p.kill()
    return out


def test_values_only_allreduce_world2():
    out = _run(_worker_allreduce)
    assert out == {0: True, 1: True}, out


def test_topology_broadcast_and_checksum_world2():
    out = _run(_worker_broadcast)
    assert out == {0: True, 1: True}, out


def test_rank_leaving_before_collective_raises_on_survivor():
    out = _run(_worker_rank_fails)
    assert out[1] == "left"
    assert out[0].startswith("raised"), out
