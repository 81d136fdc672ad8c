"""C-ABI argument validation: every entry point rejects bad arguments with
SL_ERR_INVALID / SL_ERR_UNSUPPORTED and a message, before any device work
(so these run without a GPU).  Messages that the reference raises as
ValueError keep its wording (csrc/bindings.cpp:208-225)."""
import ctypes

import pytest

from sparsecore_b200 import _native as N

BAD = N.P(1)  # a non-NULL stand-in; never dereferenced on these paths


@pytest.fixture(scope="module")
def lib():
    from sparsecore_b200.build import build

    build()
    return N.load_library()


def csr(nrows=4, ncols=5, cap=8, null_rows=False, null_slots=False):
    p = 0 if null_rows else 1
    q = 0 if null_slots else 1
    return N.SlCsr(nrows, ncols, cap, q, q, p, p, p)


def err(lib):
    return lib.sl_last_error().decode()


def test_spmm_and_sddmm_validation(lib):
    ref = ctypes.byref
    assert lib.sl_spmm_fwd(None, BAD, 5, 3, BAD, None) == N.SL_ERR_INVALID
    assert "W is NULL" in err(lib)
    assert lib.sl_spmm_fwd(ref(csr()), BAD, 6, 3, BAD, None) == N.SL_ERR_INVALID
    assert "Inner dimensions must match for matmul" in err(lib)
    assert lib.sl_spmm_fwd(ref(csr()), BAD, 5, -1, BAD, None) == N.SL_ERR_INVALID
    assert lib.sl_spmm_fwd(ref(csr()), None, 5, 3, BAD, None) == N.SL_ERR_INVALID
    assert lib.sl_spmm_fwd(ref(csr(null_rows=True)), BAD, 5, 3, BAD, None) == N.SL_ERR_INVALID
    assert "NULL row array" in err(lib)
    assert lib.sl_spmm_fwd(ref(csr(null_slots=True)), BAD, 5, 3, BAD, None) == N.SL_ERR_INVALID
    assert lib.sl_spmm_fwd(ref(N.SlCsr(-1, 5, 0, 1, 1, 1, 1, 1)), BAD, 5, 3, BAD, None) == N.SL_ERR_INVALID
    big = N.SlCsr(1 << 32, 5, 8, 1, 1, 1, 1, 1)
    assert lib.sl_spmm_fwd(ref(big), BAD, 5, 3, BAD, None) == N.SL_ERR_UNSUPPORTED
    assert lib.sl_sddmm_dw(ref(csr()), BAD, BAD, -2, BAD, None) == N.SL_ERR_INVALID
    assert lib.sl_sddmm_dw(ref(csr()), BAD, BAD, 3, None, None) == N.SL_ERR_INVALID
    assert lib.sl_sddmm_dw(ref(csr()), None, BAD, 3, BAD, None) == N.SL_ERR_INVALID


def test_fused_epilogue_and_bias_transpose_validation(lib):
    ref = ctypes.byref
    # activation code out of range; an activation without H
    assert lib.sl_spmm_fwd_act(ref(csr()), BAD, 5, 3, None, 3, BAD, BAD, None) == N.SL_ERR_INVALID
    assert "act must be" in err(lib)
    assert lib.sl_spmm_fwd_act(ref(csr()), BAD, 5, 3, None, 2, BAD, None, None) == N.SL_ERR_INVALID
    assert "NULL H" in err(lib)
    assert lib.sl_spmm_fwd_act(ref(csr()), BAD, 6, 3, None, 0, BAD, None, None) == N.SL_ERR_INVALID
    assert "Inner dimensions must match for matmul" in err(lib)
    assert lib.sl_spmm_fwd_gelu(ref(csr()), BAD, 5, 3, BAD, None, None) == N.SL_ERR_INVALID
    # the bias transpose: NULL bias, in place, negative shape
    assert lib.sl_transpose_bias_f32(BAD, 4, 4, None, N.P(2), None) == N.SL_ERR_INVALID
    assert "NULL bias" in err(lib)
    assert lib.sl_transpose_bias_f32(BAD, 4, 4, BAD, BAD, None) == N.SL_ERR_INVALID
    assert lib.sl_transpose_bias_f32(BAD, -1, 4, BAD, N.P(2), None) == N.SL_ERR_INVALID


def test_layout_and_transpose_validation(lib):
    ref = ctypes.byref
    assert lib.sl_transpose_count(ref(csr(ncols=100000)), 1.2, BAD, BAD, BAD, BAD, BAD, None) \
        == N.SL_ERR_UNSUPPORTED
    assert lib.sl_transpose_count(ref(csr()), 0.5, BAD, BAD, BAD, BAD, BAD, None) == N.SL_ERR_INVALID
    assert "padding_ratio" in err(lib)
    assert lib.sl_transpose_count(ref(csr()), 1.2, BAD, BAD, BAD, BAD, None, None) == N.SL_ERR_INVALID
    assert "scratch" in err(lib)
    WT = N.SlCsr(4, 4, 8, 1, 1, 1, 1, 1)  # wrong shape for csr() (4 x 5)
    assert lib.sl_transpose_fill(ref(csr()), ref(WT), BAD, BAD, None) == N.SL_ERR_INVALID
    assert lib.sl_values_gather(BAD, BAD, BAD, -1, None) == N.SL_ERR_INVALID
    assert lib.sl_values_gather(None, BAD, BAD, 4, None) == N.SL_ERR_INVALID
    assert lib.sl_dense_count(BAD, -1, 3, 0.0, 1.2, BAD, BAD, BAD, BAD, None) == N.SL_ERR_INVALID
    assert lib.sl_dense_count(None, 3, 3, 0.0, 1.2, BAD, BAD, BAD, BAD, None) == N.SL_ERR_INVALID
    assert lib.sl_dense_fill(None, 0.0, ref(csr()), None) == N.SL_ERR_INVALID
    assert lib.sl_to_dense(ref(csr()), None, None) == N.SL_ERR_INVALID
    assert lib.sl_check_invariants(ref(csr()), 8, None, None) == N.SL_ERR_INVALID
    assert lib.sl_capacity_scan(BAD, 3, 0.9, BAD, BAD, BAD, None) == N.SL_ERR_INVALID
    assert lib.sl_capacity_scan(None, 3, 1.2, BAD, BAD, BAD, None) == N.SL_ERR_INVALID
    assert lib.sl_exclusive_scan(BAD, -3, BAD, BAD, None) == N.SL_ERR_INVALID
    assert lib.sl_exclusive_scan(None, 3, BAD, BAD, None) == N.SL_ERR_INVALID
    assert lib.sl_transpose_f32(BAD, -1, 2, BAD, None) == N.SL_ERR_INVALID
    assert lib.sl_transpose_f32(BAD, 2, 2, BAD, None) == N.SL_ERR_INVALID
    assert "in-place" in err(lib)
    assert lib.sl_transpose_f32(None, 2, 2, N.P(2), None) == N.SL_ERR_INVALID


def test_router_and_dp_validation(lib):
    ref = ctypes.byref
    assert lib.sl_dst_threshold(ref(csr()), 0, BAD, BAD, None) == N.SL_ERR_INVALID
    assert lib.sl_dst_threshold(ref(csr()), 3, BAD, None, None) == N.SL_ERR_INVALID
    assert lib.sl_dst_keep(ref(csr()), None, BAD, BAD, None) == N.SL_ERR_INVALID
    wide = csr(ncols=int(lib.sl_dst_max_ncols()) + 1)
    assert lib.sl_dst_apply_random(ref(wide), BAD, BAD, BAD, BAD, None) == N.SL_ERR_UNSUPPORTED
    assert lib.sl_dst_apply_random(ref(csr()), BAD, BAD, None, BAD, None) == N.SL_ERR_INVALID
    assert lib.sl_dst_apply_topk(ref(csr()), BAD, BAD, None, BAD, None) == N.SL_ERR_INVALID
    assert lib.sl_dst_apply_cols(ref(csr()), BAD, BAD, None, BAD, BAD, None) == N.SL_ERR_INVALID
    assert lib.sl_dense_grad(BAD, BAD, -1, 2, 2, BAD, None) == N.SL_ERR_INVALID
    assert lib.sl_dense_grad(BAD, BAD, 2, 2, 2, None, None) == N.SL_ERR_INVALID
    assert lib.sl_dense_grad(BAD, None, 2, 2, 2, BAD, None) == N.SL_ERR_INVALID
    assert lib.sl_pack_live(ref(csr()), None, BAD, BAD, None) == N.SL_ERR_INVALID
    assert lib.sl_unpack_live(ref(csr()), BAD, None, BAD, 1.0, None) == N.SL_ERR_INVALID
    # host-only SET draws: NULL state / arrays, survivors out of range, short buffer
    import numpy as np

    st = np.zeros(4, np.uint64)
    h32 = np.zeros(1, np.int32)
    u32 = np.zeros(1, np.uint32)
    live, keep = np.array([5], np.int32), np.array([6], np.int32)
    cnt, rk, nr = np.zeros(1, np.int32), np.zeros(4, np.int32), np.zeros(1, np.int64)
    a = lambda x: x.ctypes.data_as(ctypes.c_void_p)  # noqa: E731
    assert lib.sl_set_regrow_draws(None, a(h32), a(u32), 1, a(live), a(keep), 10, a(cnt), a(rk), 4,
                                   a(nr)) == N.SL_ERR_INVALID
    assert lib.sl_set_regrow_draws(a(st), a(h32), a(u32), 1, None, a(keep), 10, a(cnt), a(rk), 4,
                                   a(nr)) == N.SL_ERR_INVALID
    assert lib.sl_set_regrow_draws(a(st), a(h32), a(u32), 1, a(live), a(keep), 10, a(cnt), a(rk), 4,
                                   a(nr)) == N.SL_ERR_INVALID
    assert "survivors out of range" in err(lib)
    keep[0] = 1
    assert lib.sl_set_regrow_draws(a(st), a(h32), a(u32), 1, a(live), a(keep), 10, a(cnt), a(rk), 3,
                                   a(nr)) == N.SL_ERR_INVALID
    assert "too small" in err(lib)


def test_python_layer_maps_codes_to_reference_exceptions(lib):
    N._lib = lib
    try:
        with pytest.raises(ValueError, match="Inner dimensions must match"):
            N.call("sl_spmm_fwd", ctypes.byref(csr()), BAD, 6, 3, BAD, None)
        big = N.SlCsr(1 << 32, 5, 8, 1, 1, 1, 1, 1)
        with pytest.raises(RuntimeError, match="int32"):
            N.call("sl_spmm_fwd", ctypes.byref(big), BAD, 5, 3, BAD, None)
    finally:
        N._lib = None
