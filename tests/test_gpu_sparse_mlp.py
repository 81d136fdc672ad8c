"""sparse_mlp (two SparseLinears with the hidden activation kept in the
kernels' layout, fc1's bias and the activation in the forward kernel's
epilogue, fc2's bias in the output transpose) equals the unfused module
composition bit for bit: output, input gradient, both weight gradients and
both bias gradients; with and without the side-stream weight gradient."""
import pytest
import torch

from gpu_helpers import bits_equal, dev

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("act", ["gelu", "relu"])
@pytest.mark.parametrize("async_dw", [False, True])
@pytest.mark.parametrize("bias", [(False, False), (True, True), (True, False), (False, True)])
@pytest.mark.parametrize("T", [37, 300])
def test_sparse_mlp_matches_unfused(act, async_dw, bias, T):
    import sparsecore_b200 as sl
    from sparsecore_b200 import ops

    torch.manual_seed(3)
    fc1 = sl.SparseLinear(96, 160, bias=bias[0], sparsity=0.85)
    fc2 = sl.SparseLinear(160, 48, bias=bias[1], sparsity=0.7)
    x = torch.randn(5, T, 96, device=dev())
    gy = torch.randn(5, T, 48, device=dev())
    f = torch.nn.functional.gelu if act == "gelu" else torch.relu
    params = [fc1._values, fc2._values] + [b for b in (fc1.bias, fc2.bias) if b is not None]

    xa = x.clone().requires_grad_(True)
    ya = fc2(f(fc1(xa)))
    ya.backward(gy)
    ref = (ya.detach(), xa.grad) + tuple(p.grad.clone() for p in params)
    for p in params:
        p.grad = None

    ops.set_async_weight_grad(async_dw)
    try:
        xb = x.clone().requires_grad_(True)
        yb = sl.sparse_mlp(xb, fc1, fc2, act)
        yb.backward(gy)
        torch.cuda.synchronize()
    finally:
        ops.set_async_weight_grad(False)
    got = (yb.detach(), xb.grad) + tuple(p.grad for p in params)
    names = ["y", "dx", "dW1", "dW2", "db1", "db2"]
    for a, b, n in zip(got, ref, names):
        assert bits_equal(a, b), n


def test_sparse_mlp_rejects_unknown_activation():
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


@pytest.mark.parametrize("N,path", [(1, None), (32, None), (185, None), (256, "rows"),
                                    (1024, "xs"), (1024, None)])
@pytest.mark.parametrize("act", [0, 1, 2])
@pytest.mark.parametrize("with_bias", [True, False])
def test_fused_bias_act_epilogue_equals_torch(N, path, act, with_bias, monkeypatch):
    """sl_spmm_fwd_act: Y equals sl_spmm_fwd's plus torch's broadcast bias add,
    and H torch's ReLU / exact GELU of Y, bit for bit, on the fused epilogues
    (row-gather, X-stationary) and the second pass (small N)."""
    import sparsecore_b200 as sl
    from sparsecore_b200 import _native as N_
    from sparsecore_b200 import ops

    if path is not None:
        monkeypatch.setenv("SPARSECORE_B200_FWD", path)
    g = torch.Generator().manual_seed(N + act)
    W = sl.PaddedCSR.random(300, 700, sparsity=0.8, seed=N)
    X = (torch.randn(700, N, generator=g) * 3.0).to(dev())
    b = (torch.randn(300, generator=g) * 2.0).to(dev()) if with_bias else None
    Y = torch.empty(300, N, device=dev())
    H = torch.empty(300, N, device=dev())
    N_.call("sl_spmm_fwd_act", W._abi_ref(), N_.ptr(X), 700, N, N_.ptr(b), act, N_.ptr(Y),
            N_.ptr(H), W._stream())
    ref = ops._spmm_raw(W, X)
    if with_bias:
        ref = (ref.t() + b).t()
    assert bits_equal(Y, ref)
    if act == 1:
        assert bits_equal(H, torch.relu(ref))
    elif act == 2:
        assert bits_equal(H, torch.nn.functional.gelu(ref))
