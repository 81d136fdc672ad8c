"""GPU: PaddedCSR construction, invariants, rewrite_row, factories, the
transpose cache (mirrors the intent of the reference's test_padded_csr*.py,
test_transpose_cache.py)."""
import numpy as np
import pytest
import torch

from gpu_helpers import dev, host

pytestmark = pytest.mark.gpu


def small():
    # 3x5: row0 {1,3}, row1 {}, row2 {0,2,4}; capacities 3,1,4
    return dict(values=[1.0, 2.0, 0.0, 0.0, 3.0, 4.0, 5.0, 0.0],
                col_indices=[1, 3, -1, -1, 0, 2, 4, -1],
                row_start=[0, 3, 4], row_nnz=[2, 0, 3], row_capacity=[3, 1, 4])


def test_full_constructor_and_properties():
    import sparsecore_b200 as sl

    W = sl.PaddedCSR(3, 5, **small())
    assert W.shape == (3, 5) and W.nrows == 3 and W.ncols == 5
    assert W.nnz == 5 and W.total_capacity == 8 and W.padding_slots == 3
    assert abs(W.sparsity - (1 - 5 / 15)) < 1e-12
    assert W.topology_version == 0
    assert repr(W) == "PaddedCSR(nrows=3, ncols=5, nnz=5, capacity=8)"
    assert W.values.is_cuda and W.values.dtype == torch.float32
    assert W.col_indices.dtype == torch.int32
    D = W.to_dense().cpu()
    assert D[0, 1] == 1 and D[0, 3] == 2 and D[2, 4] == 5 and D.sum() == 15
    W.assert_invariants()
    E = sl.PaddedCSR(4, 3)
    assert E.nnz == 0 and E.total_capacity == 0 and E.sparsity == 1.0
    assert sl.PaddedCSR(0, 0).sparsity == 1.0


@pytest.mark.parametrize("mutate,msg", [
    (lambda a: a["row_start"].__setitem__(0, 1), "Invariant 3 violated: row_start[0] must be 0, got 1."),
    (lambda a: a["row_start"].__setitem__(2, 5), "Invariant 3 violated: row_start[2]=5 should equal row_start[1] + row_capacity[1] = 4."),
    (lambda a: a["row_nnz"].__setitem__(1, 2), "Invariant 4 violated at row 1: row_nnz=2 must be in [0, 1]."),
    (lambda a: a["col_indices"].__setitem__(5, 9), "Invariant 6 violated at row 2, slot 1: col_indices=9 must be in [0, 5)."),
    (lambda a: a["col_indices"].__setitem__(5, 0), "Invariant 6 violated at row 2, slot 1: col_indices=0 must be strictly greater than previous=0"),
    (lambda a: a["col_indices"].__setitem__(2, 4), "Invariants 5+7 violated at row 0, slot 2: padding col_indices=4 must be -1."),
    (lambda a: a["values"].append(0.0), "Invariant 2 violated: values (9) and col_indices (8) must have the same length."),
    (lambda a: a["row_capacity"].__setitem__(2, 5), "Invariant 2 violated: values.size()=8 does not match total_capacity=9"),
    (lambda a: a["row_nnz"].pop(), "Metadata array length mismatch"),
])
def test_invariant_violations_raise(mutate, msg):
    import sparsecore_b200 as sl

    a = small()
    mutate(a)
    with pytest.raises(ValueError) as ei:
        sl.PaddedCSR(3, 5, **a)
    assert "PaddedCSR invariant check failed: " in str(ei.value)
    assert msg in str(ei.value)


def test_rewrite_row_semantics_and_errors():
    import sparsecore_b200 as sl

    W = sl.PaddedCSR(3, 5, **small())
    W.rewrite_row(2, np.array([1, 3], np.int32), np.array([7.0, 8.0], np.float32))
    assert W.topology_version == 1 and W.nnz == 4
    assert host(W.col_indices)[4:8].tolist() == [1, 3, -1, -1]
    assert host(W.values)[4:8].tolist() == [7.0, 8.0, 0.0, 0.0]
    assert host(W.row_nnz).tolist() == [2, 0, 2]
    W.assert_invariants()
    W.rewrite_row(1, [4], [9.0])
    assert W.nnz == 5 and W.topology_version == 2
    for args, msg in [((3, [0], [1.0]), "out of range [0, 3)"),
                      ((0, [0, 1], [1.0]), "must equal new_values.size()"),
                      ((1, [0, 1], [1.0, 2.0]), "has capacity 1 but got 2"),
                      ((0, [2, 1], [1.0, 2.0]), "strictly ascending"),
                      ((0, [5], [1.0]), "new_cols[0]=5 out of range [0, 5)")]:
        with pytest.raises(ValueError, match=msg.replace("[", r"\[").replace("(", r"\(").replace(")", r"\)")):
            W.rewrite_row(*args)
    assert W.topology_version == 2


def test_from_dense_threshold_and_roundtrip():
    import sparsecore_b200 as sl

    g = torch.Generator().manual_seed(0)
    D = torch.randn(40, 70, generator=g)
    D[torch.rand(40, 70, generator=g) < 0.8] = 0
    D[3] = 0  # empty row
    W = sl.PaddedCSR.from_dense(D)
    assert torch.equal(W.to_dense().cpu(), D)
    caps = host(W.row_capacity)
    nnz = host(W.row_nnz)
    assert np.array_equal(caps, np.maximum(1, np.ceil(nnz * 1.2)).astype(np.int32))
    Wt = sl.PaddedCSR.from_dense(D, threshold=0.5)
    assert torch.equal(Wt.to_dense().cpu(), torch.where(D.abs() > 0.5, D, torch.zeros_like(D)))
    W0 = sl.PaddedCSR.from_dense(D, padding_ratio=0.0)
    assert W0.padding_slots == 1  # only the empty row's floor-of-1 slot
    with pytest.raises(ValueError):
        sl.PaddedCSR.from_dense(torch.zeros(3))
    with pytest.raises(ValueError):
        sl.PaddedCSR.from_dense(D, padding_ratio=-0.5)


def test_from_torch_sparse_csr_matches_from_dense():
    import sparsecore_b200 as sl

    W1 = sl.PaddedCSR.random(50, 60, sparsity=0.8, seed=4)
    D = W1.to_dense().cpu()
    W2 = sl.PaddedCSR.from_torch_sparse_csr(D.to_sparse_csr())
    for a in ("values", "col_indices", "row_start", "row_nnz", "row_capacity"):
        assert torch.equal(getattr(W1, a), getattr(W2, a)), a
    with pytest.raises(ValueError):
        sl.PaddedCSR.from_torch_sparse_csr(D)
    with pytest.raises(ValueError):
        sl.PaddedCSR.random(3, 3, sparsity=1.0)


def test_transpose_cache_hit_miss_refresh():
    import sparsecore_b200 as sl
    from sparsecore_b200.ops import _cached_transpose, _clear_transpose_cache, _transpose_cache

    _clear_transpose_cache()
    W = sl.PaddedCSR.random(30, 20, sparsity=0.7, seed=1)
    WT1 = _cached_transpose(W)
    assert len(_transpose_cache) == 1
    WT2 = _cached_transpose(W)
    assert WT2 is WT1  # hit
    W.values.mul_(2.0)  # optimizer-style in-place update
    WT3 = _cached_transpose(W)
    assert WT3 is WT1
    assert torch.equal(WT3.to_dense(), W.to_dense().t())  # refreshed values
    s0 = int(host(W.row_start)[0])
    n0 = int(host(W.row_nnz)[0])
    cols = host(W.col_indices)[s0:s0 + n0][:-1] if n0 else np.zeros(0, np.int32)
    W.rewrite_row(0, cols, np.ones(cols.size, np.float32))
    WT4 = _cached_transpose(W)
    assert WT4 is not WT1  # topology changed -> rebuilt
    assert torch.equal(WT4.to_dense(), W.to_dense().t())
    key = id(W)
    del W, WT1, WT2, WT3, WT4
    import gc

    gc.collect()
    assert key not in _transpose_cache  # dropped with W
    _clear_transpose_cache()


def test_spmm_validation_errors():
    import sparsecore_b200 as sl

    W = sl.PaddedCSR.random(4, 6, sparsity=0.5, seed=0)
    with pytest.raises(TypeError):
        sl.spmm("W", torch.zeros(6, 2, device=dev()))
    with pytest.raises(TypeError):
        sl.spmm(W, np.zeros((6, 2), np.float32))
    with pytest.raises(RuntimeError):
        sl.spmm(W, torch.zeros(6, 2))  # CPU tensor: no CPU path
    with pytest.raises(ValueError):
        sl.spmm(W, torch.zeros(6, device=dev()))
    with pytest.raises(ValueError):
        sl.spmm(W, torch.zeros(5, 2, device=dev()))
    with pytest.raises(ValueError):
        sl.spmm(W, torch.zeros(6, 2, device=dev()), kernel="nope")
    for k in ("auto", "simd", "scalar"):
        assert sl.spmm(W, torch.ones(6, 2, device=dev()), kernel=k).shape == (4, 2)
    # fp64 input is coerced to fp32
    assert sl.spmm(W, torch.ones(6, 2, device=dev(), dtype=torch.float64)).dtype == torch.float32


def test_dense_transpose_kernel_exact():
    """sl_transpose_f32 (SparseLinear's layout change) is an exact copy."""
    from sparsecore_b200 import ops

    g = torch.Generator().manual_seed(5)
    # scalar path (odd shapes) and the 64 x 64 float4 path, whole and partial tiles
    for r, c in [(1, 1), (33, 65), (1000, 7), (7, 1000), (512, 3072), (68, 132), (4, 200), (260, 4)]:
        a = torch.randn(r, c, generator=g).cuda()
        assert torch.equal(ops._transpose(a), a.t().contiguous()), (r, c)


def test_transpose_with_bias_matches_torch_add():
    """sl_transpose_bias_f32 (the SparseLinear output transpose with the bias
    add fused in) equals torch's transpose followed by ``+ bias`` bit for bit,
    on the scalar path (odd shapes) and the float4 path."""
    from sparsecore_b200 import ops

    from gpu_helpers import bits_equal

    g = torch.Generator().manual_seed(6)
    for r, c in [(1, 1), (33, 65), (1000, 7), (512, 3072), (68, 132), (260, 4)]:
        a = torch.randn(r, c, generator=g).cuda()
        b = torch.randn(r, generator=g).cuda()
        assert bits_equal(ops._transpose_bias(a, b), a.t().contiguous() + b), (r, c)


@pytest.mark.parametrize("T,fin,fout", [(37, 96, 48), (256, 384, 1152), (130, 99, 77)])
def test_sparse_linear_fused_bias_matches_unfused(T, fin, fout):
    """A SparseLinear with a bias (its output transpose adds the bias) gives
    the same output and gradients, bit for bit, as the bias-free layer plus
    torch's broadcast add: y, dx, dW and dbias."""
    import sparsecore_b200 as sl
    from sparsecore_b200.ops import _SparseLinearFunction

    from gpu_helpers import bits_equal

    torch.manual_seed(T)
    layer = sl.SparseLinear(fin, fout, sparsity=0.8, bias=True, device=dev())
    x = torch.randn(T, fin, device=dev())
    gy = torch.randn(T, fout, device=dev())
    x1 = x.clone().requires_grad_(True)
    y1 = layer(x1)
    y1.backward(gy)
    g1 = (y1.detach(), x1.grad, layer._values.grad.clone(), layer.bias.grad.clone())
    layer.zero_grad(set_to_none=True)
    x2 = x.clone().requires_grad_(True)
    y2 = _SparseLinearFunction.apply(layer._values, layer._csr, x2) + layer.bias
    y2.backward(gy)
    torch.cuda.synchronize()
    g2 = (y2.detach(), x2.grad, layer._values.grad, layer.bias.grad)
    for a, b, name in zip(g1, g2, ("y", "dx", "dW", "dbias")):
        assert bits_equal(a, b), name
