"""sparse_mlp (two SparseLinears with the hidden activation kept in the
kernels' layout) equals the unfused module composition bit for bit: output,
input gradient and both weight gradients; with and without the side-stream
weight gradient."""
import pytest
import torch

from gpu_helpers import bits_equal, dev

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("act", ["gelu", "relu"])
@pytest.mark.parametrize("async_dw", [False, True])
def test_sparse_mlp_matches_unfused(act, async_dw):
    import sparsecore_b200 as sl
    from sparsecore_b200 import ops

    torch.manual_seed(3)
    fc1 = sl.SparseLinear(96, 160, bias=False, sparsity=0.85)
    fc2 = sl.SparseLinear(160, 48, bias=False, sparsity=0.7)
    x = torch.randn(5, 37, 96, device=dev())
    gy = torch.randn(5, 37, 48, device=dev())
    f = torch.nn.functional.gelu if act == "gelu" else torch.relu

    xa = x.clone().requires_grad_(True)
    ya = fc2(f(fc1(xa)))
    ya.backward(gy)
    ref = (ya.detach(), xa.grad, fc1._values.grad.clone(), fc2._values.grad.clone())
    fc1._values.grad = None
    fc2._values.grad = None

    ops.set_async_weight_grad(async_dw)
    try:
        xb = x.clone().requires_grad_(True)
        yb = sl.sparse_mlp(xb, fc1, fc2, act)
        yb.backward(gy)
        torch.cuda.synchronize()
    finally:
        ops.set_async_weight_grad(False)
    assert bits_equal(yb, ref[0])
    assert bits_equal(xb.grad, ref[1])
    assert bits_equal(fc1._values.grad, ref[2])
    assert bits_equal(fc2._values.grad, ref[3])


def test_sparse_mlp_falls_back_with_bias_or_hooks():
    import sparsecore_b200 as sl

    torch.manual_seed(4)
    fc1 = sl.SparseLinear(16, 24, bias=True, sparsity=0.5)
    fc2 = sl.SparseLinear(24, 8, bias=False, sparsity=0.5)
    x = torch.randn(6, 16, device=dev())
    assert torch.equal(sl.sparse_mlp(x, fc1, fc2, "relu"), fc2(torch.relu(fc1(x))))
    with pytest.raises(ValueError):
        sl.sparse_mlp(x, fc1, fc2, "tanh")


@pytest.mark.parametrize("N,path", [(1, None), (8, None), (32, None), (185, None), (256, "rows"),
                                    (1024, "xs"), (1024, None)])
def test_fused_gelu_epilogue_equals_torch_gelu(N, path, monkeypatch):
    """sl_spmm_fwd_gelu: Y equals sl_spmm_fwd's and H equals torch's exact
    GELU of Y bit for bit, on the fused epilogues (row-gather, X-stationary)
    and the second-pass kernel (small N); values span the GELU's range."""
    import sparsecore_b200 as sl
    from sparsecore_b200 import ops

    if path is not None:
        monkeypatch.setenv("SPARSECORE_B200_FWD", path)
    g = torch.Generator().manual_seed(N)
    W = sl.PaddedCSR.random(300, 700, sparsity=0.8, seed=N)
    X = (torch.randn(700, N, generator=g) * 3.0).to(dev())
    Y, H = ops._spmm_gelu_raw(W, X)
    assert bits_equal(Y, ops._spmm_raw(W, X))
    assert bits_equal(H, torch.nn.functional.gelu(Y))
