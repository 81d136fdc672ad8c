"""ctypes binding of the sparsecore_b200 C ABI (include/sparsecore_b200.h).

The CUDA library is the only compute path: there is no CPU fallback.  If the
library is missing or no CUDA device is present, every compute entry point
raises RuntimeError.
"""
from __future__ import annotations

import ctypes
import os
import threading

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "_lib", "libsparsecore_b200.so")

SL_OK, SL_ERR_INVALID, SL_ERR_CUDA, SL_ERR_UNSUPPORTED, SL_ERR_TIMEOUT = 0, 1, 2, 3, 4

P = ctypes.c_void_p
I64 = ctypes.c_int64
I32 = ctypes.c_int
F32 = ctypes.c_float
F64 = ctypes.c_double


class SlCsr(ctypes.Structure):
    """Mirror of `sl_csr` (device pointers)."""

    _fields_ = [
        ("nrows", I64),
        ("ncols", I64),
        ("total_capacity", I64),
        ("values", P),
        ("col_indices", P),
        ("row_start", P),
        ("row_nnz", P),
        ("row_capacity", P),
    ]


# name -> (restype, argtypes); every symbol the header declares.
SIGNATURES: dict[str, tuple] = {
    "sl_last_error": (ctypes.c_char_p, []),
    "sl_version": (ctypes.c_char_p, []),
    "sl_last_kernel": (ctypes.c_char_p, []),
    "sl_probe_threads": (I64, []),
    "sl_probe_ffma": (I32, [I64, P, P]),
    "sl_probe_smem": (I32, [I64, P, P]),
    "sl_device_status": (I32, [I32, P]),
    "sl_selftest_bounded_wait": (I32, [I64, P]),
    "sl_spmm_fwd": (I32, [P, P, I64, I64, P, P]),
    "sl_spmm_fwd_gelu": (I32, [P, P, I64, I64, P, P, P]),
    "sl_spmm_fwd_act": (I32, [P, P, I64, I64, P, I32, P, P, P]),
    "sl_sddmm_dw": (I32, [P, P, P, I64, P, P]),
    "sl_transpose_scratch_bytes": (I64, [I64, I64]),
    "sl_transpose_count": (I32, [P, F64, P, P, P, P, P, P]),
    "sl_transpose_fill": (I32, [P, P, P, P, P]),
    "sl_values_gather": (I32, [P, P, P, I64, P]),
    "sl_transpose_with_perm_noalloc": (I32, [P, F64, P, P, P, P]),
    "sl_dense_count": (I32, [P, I64, I64, F32, F64, P, P, P, P, P]),
    "sl_dense_fill": (I32, [P, F32, P, P]),
    "sl_capacity_scan": (I32, [P, I64, F64, P, P, P, P]),
    "sl_to_dense": (I32, [P, P, P]),
    "sl_check_invariants": (I32, [P, I64, P, P]),
    "sl_dense_grad": (I32, [P, P, I64, I64, I64, P, P]),
    "sl_rigl_prep": (I32, [P, P, P, P, P, P]),
    "sl_rigl_tile_cols": (I64, [I64, I64]),
    "sl_rigl_candidates": (I32, [P, P, I64, I64, I64, P, P, I64, I64, P, P, P, P, P]),
    "sl_rigl_merge": (I32, [I64, I64, I64, I64, P, P, P, P, P, P, P, P, P, P]),
    "sl_dst_scratch_bytes": (I64, []),
    "sl_dst_max_ncols": (I64, []),
    "sl_dst_threshold": (I32, [P, I64, P, P, P]),
    "sl_dst_keep": (I32, [P, P, P, P, P]),
    "sl_dst_apply_random": (I32, [P, P, P, P, P, P]),
    "sl_dst_apply_topk": (I32, [P, P, P, P, P, P]),
    "sl_dst_apply_cols": (I32, [P, P, P, P, P, P, P]),
    "sl_pack_live": (I32, [P, P, P, P, P]),
    "sl_adamw_live": (I32, [P, P, P, P, F32, F32, F32, F32, F32, I64, P]),
    "sl_unpack_live": (I32, [P, P, P, P, F32, P]),
    "sl_exclusive_scan": (I32, [P, I64, P, P, P]),
    "sl_pack_live_batch": (I32, [P, I64, I64, P, P]),
    "sl_unpack_live_batch": (I32, [P, I64, I64, P, P]),
    "sl_transpose_f32": (I32, [P, I64, I64, P, P]),
    "sl_transpose_bias_f32": (I32, [P, I64, I64, P, P, P]),
    "sl_set_regrow_draws": (I32, [P, P, P, I64, P, P, I64, P, P, I64, P]),
}

_lib = None
_lock = threading.Lock()


def load_library(path: str = LIB_PATH) -> ctypes.CDLL:
    """Load the library without requiring a GPU (used by CPU-side tests)."""
    lib = ctypes.CDLL(path)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not os.path.exists(LIB_PATH):
                    raise RuntimeError(
                        "sparsecore_b200: CUDA library not built (expected "
                        f"{LIB_PATH}); run `python -m sparsecore_b200.build`. "
                        "There is no CPU fallback.")
                _lib = load_library()
    return _lib


def require_cuda(device: torch.device | None = None) -> torch.device:
    if not torch.cuda.is_available():
        raise RuntimeError(
            "sparsecore_b200 requires a CUDA device (B200 / sm_100a); there is no CPU path.")
    if device is None:
        return torch.device("cuda", torch.cuda.current_device())
    device = torch.device(device)
    if device.type != "cuda":
        raise RuntimeError(f"sparsecore_b200 tensors live on CUDA devices, got device={device}")
    if device.index is None:
        device = torch.device("cuda", torch.cuda.current_device())
    return device


_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def stream_ptr(device: torch.device) -> P:
    """The current CUDA stream of `device` (the capture stream under graph
    capture) as a raw pointer; the direct query costs about 1 us, the
    torch.cuda.current_stream object about 9."""
    if _raw_stream is not None and device.index is not None:
        return P(_raw_stream(device.index))
    return P(torch.cuda.current_stream(device).cuda_stream)


def ptr(t: torch.Tensor | None) -> P:
    return P(t.data_ptr()) if t is not None else P(0)


# Kernels each entry point launches (for launch accounting).
KERNELS_PER_CALL = {
    "sl_spmm_fwd": 1, "sl_spmm_fwd_gelu": 1, "sl_spmm_fwd_act": 1, "sl_transpose_bias_f32": 1, "sl_sddmm_dw": 1, "sl_transpose_count": 3, "sl_transpose_fill": 2,
    "sl_transpose_with_perm_noalloc": 5,
    "sl_values_gather": 1, "sl_dense_count": 2, "sl_dense_fill": 1, "sl_capacity_scan": 1,
    "sl_to_dense": 1, "sl_check_invariants": 2, "sl_dense_grad": 1, "sl_rigl_prep": 1, "sl_rigl_candidates": 1, "sl_rigl_merge": 1, "sl_dst_threshold": 9,
    "sl_dst_keep": 1, "sl_dst_apply_random": 1, "sl_dst_apply_topk": 1, "sl_dst_apply_cols": 1,
    "sl_pack_live": 1, "sl_unpack_live": 1, "sl_adamw_live": 1, "sl_pack_live_batch": 1,
    "sl_unpack_live_batch": 1, "sl_exclusive_scan": 1,
    "sl_set_regrow_draws": 0,  # host only
    "sl_probe_ffma": 1, "sl_probe_smem": 1,
}
launches = {"count": 0}


_fns: dict = {}


def call(name: str, *args) -> None:
    """Invoke a status-returning entry point; raise on error; count launches."""
    lb = lib()
    fn = _fns.get((id(lb), name))
    if fn is None:
        fn = _fns[(id(lb), name)] = getattr(lb, name)
    rc = fn(*args)
    launches["count"] += KERNELS_PER_CALL.get(name, 1)
    check(rc, name)


def check(rc: int, fn: str = "") -> None:
    """Translate a C-ABI status into the reference's Python exceptions."""
    if rc == SL_OK:
        return
    msg = (lib().sl_last_error() or b"").decode("utf-8", "replace") or fn
    if rc == SL_ERR_INVALID:
        raise ValueError(msg)
    raise RuntimeError(msg)


STATUS_TIMEOUT_BIT = 1


def check_device_status(device: torch.device | int | None = None, sync: bool = True) -> None:
    """Read and clear the library's device status word; raise if a bounded
    device-side wait gave up since the last check.

    The TMA-fed kernels (X-stationary forward, tiled SDDMM) bound every
    mbarrier wait.  A wait that runs out raises bit 0 of a per-device status
    word and the kernel returns early, so its output (Y or dW) is incomplete;
    the C call itself has already returned SL_OK by then.  This check turns
    that bit into ``RuntimeError`` (the C-ABI's SL_ERR_TIMEOUT).  It costs a
    device synchronisation (``sync=True``) plus a 4-byte read, so callers run
    it where they synchronise anyway: router updates, graph re-captures, the
    end of a benchmark."""
    dev = require_cuda(None if device is None else torch.device("cuda", device)
                       if isinstance(device, int) else device)
    if sync:
        torch.cuda.synchronize(dev)
    st = ctypes.c_uint(0)
    with torch.cuda.device(dev):
        check(lib().sl_device_status(1, ctypes.byref(st)), "sl_device_status")
    if st.value & STATUS_TIMEOUT_BIT:
        raise RuntimeError(
            f"sparsecore_b200: a bounded device-side wait timed out on {dev} (status word "
            f"0x{st.value:x}, SL_ERR_TIMEOUT): the outputs of kernels launched since the last "
            "status check are incomplete")


def measure_ceilings(device: torch.device | None = None) -> dict:
    """Measured FP32 FMA and shared-memory throughput of this GPU (the
    library's probe kernels, CUDA events, best of 5 after a warm-up), for the
    roofline fractions of the FMA- and shared-memory-bound kernels."""
    dev = require_cuda(device)
    n = int(lib().sl_probe_threads())
    out = torch.empty(n, dtype=torch.float32, device=dev)
    s = stream_ptr(dev)

    def best_ms(name, iters):
        fn = getattr(lib(), name)
        check(fn(iters, ptr(out), s), name)
        torch.cuda.synchronize(dev)
        best = float("inf")
        for _ in range(5):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            check(fn(iters, ptr(out), s), name)
            b.record()
            b.synchronize()
            best = min(best, a.elapsed_time(b))
        return best

    it_f, it_s = 1 << 16, 1 << 14
    ms_f = best_ms("sl_probe_ffma", it_f)
    ms_s = best_ms("sl_probe_smem", it_s)
    fp32 = 16.0 * it_f * n / (ms_f * 1e-3) / 1e12
    smem = 32.0 * it_s * n / (ms_s * 1e-3) / 1e12
    return {"fp32_tflops": round(fp32, 2), "smem_tbs": round(smem, 2),
            "gather_ceiling_tflops": round(smem / 4.0 * 2.0, 2),
            "how": "library probe kernels (sl_probe_ffma: 8 independent FMA chains per thread; "
                   "sl_probe_smem: conflict-free 64-bit shared loads with data-dependent addresses), "
                   "64 warps per SM, "
                   "CUDA events, best of 5; gather ceiling = 4 B of shared/L1 operand per FMA"}
