"""The C-ABI compute entry points registered as torch operators
(torch.ops.sparselab.spmm_fwd / sddmm_dw): registration, fake (meta) shape
inference and the CUDA-only dispatch run on CPU; the GPU test checks that
the operators give the same bits as the library's own calls."""
import pytest
import torch

import sparsecore_b200  # noqa: F401  (registers the operators)


def _meta(n, dt=torch.int32):
    return torch.empty(n, dtype=dt, device="meta")


def test_operators_are_registered_with_fake_shapes():
    ops = torch.ops.sparselab
    Y = ops.spmm_fwd(_meta(12, torch.float32), _meta(12), _meta(4), _meta(4), _meta(4), 5,
                     torch.empty(5, 7, device="meta"))
    assert Y.shape == (4, 7) and Y.dtype == torch.float32
    dW = ops.sddmm_dw(_meta(12, torch.float32), _meta(12), _meta(4), _meta(4), _meta(4), 5,
                      torch.empty(4, 7, device="meta"), torch.empty(5, 7, device="meta"))
    assert dW.shape == (12,)


def test_cpu_tensors_have_no_kernel():
    z = lambda n, dt=torch.int32: torch.zeros(n, dtype=dt)  # noqa: E731
    with pytest.raises(NotImplementedError):
        torch.ops.sparselab.spmm_fwd(z(12, torch.float32), z(12), z(4), z(4), z(4), 5,
                                     torch.zeros(5, 7))


@pytest.mark.gpu
@pytest.mark.parametrize("N", [1, 32, 256, 2048])
def test_operators_match_the_library_calls(N):
    import sparsecore_b200 as sl
    from sparsecore_b200 import ops

    from gpu_helpers import bits_equal, dev, random_csr

    W = random_csr(700, 900, 0.1, seed=N)
    g = torch.Generator().manual_seed(N)
    X = torch.randn(900, N, generator=g).to(dev())
    dY = torch.randn(700, N, generator=g).to(dev())
    WT, _ = sl.transpose_with_perm(W)
    arr = lambda M: (M.values, M.col_indices, M.row_start, M.row_nnz, M.row_capacity, M.ncols)  # noqa: E731
    assert bits_equal(torch.ops.sparselab.spmm_fwd(*arr(W), X), ops._spmm_raw(W, X))
    assert bits_equal(torch.ops.sparselab.sddmm_dw(*arr(W), dY, X), ops._sddmm_raw(W, dY, X))
    assert bits_equal(torch.ops.sparselab.spmm_fwd(*arr(WT), dY), ops._spmm_raw(WT, dY))
