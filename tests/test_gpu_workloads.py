"""End-to-end training of the transformer workloads (configs 4 and 5, scaled
down in depth and batch) through SparseDataParallel, across a router update:
losses stay finite, every layer keeps its invariants and its Parameter alias,
the update rewrites the masks, and CUDA-graph replay of the step agrees with
eager execution."""
import dataclasses

import pytest
import torch

from gpu_helpers import dev

pytestmark = pytest.mark.gpu


def _run(cfg, steps, graph, async_dw=False):
    import sparsecore_b200 as sl
    from sparsecore_b200.dist import SparseDataParallel, sync_after_router_step
    from sparsecore_b200.graph import GraphedStep
    from sparsecore_b200.workloads import MiniGPT, lm_loss, synthetic_tokens

    from sparsecore_b200 import ops

    ops.set_async_weight_grad(async_dw)
    torch.manual_seed(0)
    model = MiniGPT(cfg, device=dev())
    algo_cls = sl.SET if cfg.router == "SET" else sl.RigL
    algo = algo_cls(sparsity=cfg.ffn_sparsity, drop_fraction=cfg.drop_fraction,
                    update_freq=cfg.update_freq, seed=0)
    model.apply(algo)
    opt = torch.optim.AdamW(model.parameters(), lr=cfg.lr, capturable=True)
    ddp = SparseDataParallel(model)
    tok = synthetic_tokens(cfg, cfg.batch, seed=5).to(dev())

    def train(t):
        opt.zero_grad(set_to_none=True)
        loss = lm_loss(model, t)
        loss.backward()
        ddp.allreduce_grads()
        opt.step()
        return loss

    layers = [m for m in model.modules() if isinstance(m, sl.SparseLinear)]
    versions0 = [m._csr.topology_version for m in layers]
    losses = [float(train(tok).item())]
    algo.step()
    sync_after_router_step(ddp, algo)
    gs = GraphedStep(model, train, (tok,)) if graph else None
    for _ in range(steps - 1):
        loss = gs() if graph else train(tok)
        losses.append(float(loss.item()))
        algo.step()
        sync_after_router_step(ddp, algo)
    ops.set_async_weight_grad(False)
    return losses, layers, versions0


@pytest.mark.parametrize("name", ["cfg4", "cfg5"])
def test_transformer_workload_trains_across_router_update(name):
    from sparsecore_b200 import workloads as W

    base = W.CFG4 if name == "cfg4" else W.CFG5
    cfg = dataclasses.replace(base, n_layers=2, batch=4, update_freq=3)
    losses, layers, v0 = _run(cfg, 5, graph=False)
    assert all(torch.isfinite(torch.tensor(losses)))
    for m, v in zip(layers, v0):
        m._csr.assert_invariants()
        assert m._values.data_ptr() == m._csr.values.data_ptr()
        assert m._csr.topology_version > v  # the update at step 3 rewrote the rows
    # Side-stream weight gradient: same values, eager and graph-replayed.
    # At ctx 512 (config 5) torch's fp32 memory-efficient attention backward
    # accumulates with atomics, so two identical runs already differ in the
    # last bits (measured: ~1e-11 in the dense gradients); config 4 (ctx 256)
    # is deterministic and must match exactly.
    overlapped, _, _ = _run(cfg, 5, graph=False, async_dw=True)
    graphed, _, _ = _run(cfg, 5, graph=True, async_dw=True)
    for other in (overlapped, graphed):
        if name == "cfg4":
            assert other == losses
        else:
            assert other == pytest.approx(losses, rel=1e-5, abs=1e-6)


def test_autograd_grad_sees_the_weight_gradient_by_default():
    """Default (synchronous) path: torch.autograd.grad and Parameter hooks see
    dW, as with the reference's _SpMMFunction."""
    import sparsecore_b200 as sl

    torch.manual_seed(0)
    layer = sl.SparseLinear(32, 16, sparsity=0.8)
    x = torch.randn(8, 32, device=dev())
    seen = []
    layer._values.register_hook(lambda g: seen.append(g.clone()))
    (gw,) = torch.autograd.grad(layer(x).square().sum(), [layer._values])
    assert gw.shape == layer._values.shape and torch.count_nonzero(gw) > 0
    assert len(seen) == 1 and torch.equal(seen[0], gw)
