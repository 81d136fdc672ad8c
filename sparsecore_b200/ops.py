"""Sparse ops: ``spmm`` and its autograd function, with the cached transpose.

Mirrors ``sparselab/ops.py``:

* ``_cached_transpose`` / ``_clear_transpose_cache`` (ops.py:66-104): W^T and
  its slot permutation are rebuilt only when ``W.topology_version`` or the
  shape changes; otherwise W^T's values are refreshed from W through the
  permutation (one gather kernel).
* ``_SpMMFunction`` (ops.py:127-210): forward Y = W.X (``sl_spmm_fwd``);
  backward dW = SDDMM(dY, X) at live slots (``sl_sddmm_dw``) and
  dX = W^T.dY (``sl_spmm_fwd`` on the cached transpose).
* ``spmm(W, X, kernel=...)`` (ops.py:217-331): same validation and error
  types; ``kernel`` accepts "auto" | "simd" | "scalar", all of which run the
  one CUDA kernel.  X must be a CUDA tensor (a CPU X raises RuntimeError:
  there is no CPU path).
"""
from __future__ import annotations

import weakref

import torch

from . import _native as N
from .layout import PaddedCSR, transpose_with_perm

__all__ = ["spmm"]

_VALID_KERNELS = ("auto", "simd", "scalar")

# id(W) -> (topology_version, (nrows, ncols), WT, perm)
_transpose_cache: dict[int, tuple] = {}


def _drop_cache_entry(key: int) -> None:
    _transpose_cache.pop(key, None)


def _cached_transpose(W: PaddedCSR) -> PaddedCSR:
    """W^T, rebuilt on topology change, value-refreshed otherwise."""
    key = id(W)
    ver = W.topology_version
    shape = (int(W.nrows), int(W.ncols))
    hit = _transpose_cache.get(key)
    if hit is not None and hit[0] == ver and hit[1] == shape:
        WT, perm = hit[2], hit[3]
        n = int(perm.numel())
        if n:
            N.call("sl_values_gather", N.ptr(perm), N.ptr(W.values), N.ptr(WT.values), n,
                                             W._stream())
        return WT
    WT, perm = transpose_with_perm(W)
    if hit is None:
        # Drop the entry when W dies, so a recycled id() can never hit.
        weakref.finalize(W, _drop_cache_entry, key)
    _transpose_cache[key] = (ver, shape, WT, perm)
    return WT


def _clear_transpose_cache() -> None:
    """Testing utility: clear all cache entries."""
    _transpose_cache.clear()


class KernelTimer:
    """Optional CUDA-event timing of every SpMM / SDDMM launch (on the stream
    the kernel is launched on), with the algorithmic bytes and FLOPs of each
    launch.  Bytes count values+indices once, the gathered dense operand once
    (K*N), the dense row operand and the output once."""

    def __init__(self):
        self.records: list[tuple] = []  # (kind, start_event, end_event, bytes, flops)

    def summary(self) -> dict:
        out: dict = {}
        for kind, e0, e1, b, f in self.records:
            d = out.setdefault(kind, {"launches": 0, "ms": 0.0, "bytes": 0, "flops": 0})
            d["launches"] += 1
            d["ms"] += e0.elapsed_time(e1)
            d["bytes"] += b
            d["flops"] += f
        return out


_timer: KernelTimer | None = None


def set_kernel_timer(t: KernelTimer | None) -> None:
    global _timer
    _timer = t


def _launch(kind, nbytes, flops, fn):
    if _timer is None:
        fn()
        return
    s = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s)
    fn()
    e1.record(s)
    _timer.records.append((kind, e0, e1, nbytes, flops))


def _spmm_raw(W: PaddedCSR, X: torch.Tensor, kind: str = "spmm_fwd") -> torch.Tensor:
    """Y = W.X on the CUDA kernel; X float32 contiguous on W's device."""
    M = W.nrows
    K, Ncol = X.shape
    Y = torch.empty(M, Ncol, dtype=torch.float32, device=X.device)
    nnz = W.nnz
    _launch(kind, 8 * nnz + 8 * M + 4 * K * Ncol + 4 * M * Ncol, 2 * nnz * Ncol,
            lambda: N.call("sl_spmm_fwd", W._abi_ref(), N.ptr(X), K, Ncol, N.ptr(Y), W._stream()))
    return Y


def _spmm_gelu_raw(W: PaddedCSR, X: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """(Y, gelu(Y)) with Y = W.X; the GELU fused into the forward kernel's
    epilogue where the decomposition allows (``sl_spmm_fwd_gelu``)."""
    M = W.nrows
    K, Ncol = X.shape
    Y = torch.empty(M, Ncol, dtype=torch.float32, device=X.device)
    H = torch.empty_like(Y)
    nnz = W.nnz
    _launch("spmm_fwd", 8 * nnz + 8 * M + 4 * K * Ncol + 8 * M * Ncol, 2 * nnz * Ncol,
            lambda: N.call("sl_spmm_fwd_gelu", W._abi_ref(), N.ptr(X), K, Ncol, N.ptr(Y), N.ptr(H),
                           W._stream()))
    return Y, H


_ACT_CODE = {"relu": 1, "gelu": 2}


def _spmm_act_raw(W: PaddedCSR, X: torch.Tensor, bias: torch.Tensor | None,
                  act: str) -> tuple[torch.Tensor, torch.Tensor]:
    """(Y, act(Y)) with Y = W.X + bias[:, None] (bias may be None); the bias
    and the activation fused into the forward kernel's epilogue where the
    decomposition allows (``sl_spmm_fwd_act``)."""
    M = W.nrows
    K, Ncol = X.shape
    Y = torch.empty(M, Ncol, dtype=torch.float32, device=X.device)
    H = torch.empty_like(Y)
    b = None if bias is None else bias.detach().to(dtype=torch.float32).contiguous()
    nnz = W.nnz
    _launch("spmm_fwd", 8 * nnz + 8 * M + 4 * K * Ncol + 8 * M * Ncol, 2 * nnz * Ncol,
            lambda: N.call("sl_spmm_fwd_act", W._abi_ref(), N.ptr(X), K, Ncol, N.ptr(b),
                           _ACT_CODE[act], N.ptr(Y), N.ptr(H), W._stream()))
    return Y, H


def _sddmm_raw(W: PaddedCSR, dY: torch.Tensor, X: torch.Tensor) -> torch.Tensor:
    """dW[total_capacity] at live slots (padding 0)."""
    dW = torch.empty(W.total_capacity, dtype=torch.float32, device=dY.device)
    M, Ncol = dY.shape
    K = X.shape[0]
    nnz = W.nnz
    _launch("sddmm_dw", 8 * nnz + 8 * M + 4 * M * Ncol + 4 * K * Ncol, 2 * nnz * Ncol,
            lambda: N.call("sl_sddmm_dw", W._abi_ref(), N.ptr(dY), N.ptr(X), Ncol, N.ptr(dW),
                           W._stream()))
    return dW


def _transpose_bias(t: torch.Tensor, bias: torch.Tensor) -> torch.Tensor:
    """[r, c] -> contiguous [c, r] with bias[r] added to every new row
    (sl_transpose_bias_f32: the layer's bias add fused into the transpose)."""
    t = t.contiguous()
    b = bias.detach().to(dtype=torch.float32).contiguous()
    r, c = t.shape
    out = torch.empty(c, r, dtype=torch.float32, device=t.device)
    _launch("transpose", 8 * r * c + 4 * r, 0,
            lambda: N.call("sl_transpose_bias_f32", N.ptr(t), r, c, N.ptr(b), N.ptr(out),
                           N.stream_ptr(t.device)))
    return out


def _transpose(t: torch.Tensor) -> torch.Tensor:
    """[r, c] fp32 CUDA tensor -> contiguous [c, r] copy (sl_transpose_f32)."""
    t = t.to(dtype=torch.float32).contiguous()
    r, c = t.shape
    out = torch.empty(c, r, dtype=torch.float32, device=t.device)
    _launch("transpose", 8 * r * c, 0,
            lambda: N.call("sl_transpose_f32", N.ptr(t), r, c, N.ptr(out), N.stream_ptr(t.device)))
    return out


def _check_dense(W: PaddedCSR, X: torch.Tensor, fn: str) -> torch.Tensor:
    if X.device.type != "cuda":
        raise RuntimeError(f"{fn}: X must be on a CUDA device (got device={X.device}). "
                           f"sparsecore_b200 has no CPU path.")
    if X.device != W.device:
        raise RuntimeError(f"{fn}: X is on {X.device} but W is on {W.device}")
    if X.dim() != 2:
        raise ValueError(f"{fn}: X must be 2-D, got ndim={X.dim()}.")
    if X.shape[0] != W.ncols:
        raise ValueError(f"{fn}: shape mismatch. W has ncols={W.ncols} but X has "
                         f"shape[0]={X.shape[0]}. Inner dimensions must match for matmul.")
    return X.to(dtype=torch.float32).contiguous()


class _SpMMFunction(torch.autograd.Function):
    """Autograd wrapper for Y = W @ X with W a PaddedCSR.

    Inputs ``(W_values, W, X, kernel)``; ``W_values`` is the tensor autograd
    tracks (it aliases ``W.values``), ``W`` travels as metadata.  Backward
    returns ``(dW_values[total_capacity], None, dX, None)``.
    """

    @staticmethod
    def forward(ctx, W_values, W, X, kernel):
        X_c = _check_dense(W, X, "spmm_simd")
        ctx.save_for_backward(W_values, X_c)
        ctx.W = W
        ctx.kernel = kernel
        return _spmm_raw(W, X_c)

    @staticmethod
    def backward(ctx, dY):
        W_values, X = ctx.saved_tensors
        W = ctx.W
        dY_c = dY.to(dtype=torch.float32).contiguous()
        if dY_c.shape[0] != W.nrows or dY_c.shape[1] != X.shape[1]:
            raise ValueError(f"spmm_grad_w_simd: dY shape {tuple(dY_c.shape)} does not match "
                             f"(W.nrows={W.nrows}, N={X.shape[1]})")
        dW = _sddmm_raw(W, dY_c, X) if ctx.needs_input_grad[0] else None
        dX = None
        if ctx.needs_input_grad[2]:
            WT = _cached_transpose(W)
            dX = _spmm_raw(WT, dY_c, kind="spmm_dx")
        return dW, None, dX, None


class _SparseLinearFunction(torch.autograd.Function):
    """Token-major form of ``_SpMMFunction`` used by ``SparseLinear``:
    ``y[T, M] = x[T, K] . W^T`` for activations laid out [tokens, features].

    The reference builds the kernels' column-per-token operand with torch
    copies (``sparselab/nn.py:229-237``: ``x.reshape(-1, in).t().contiguous()``
    and ``Y.t()`` of the result, leaving a strided output) and then adds the
    bias (``nn.py:239-241``).  Here both directions go through the transpose
    kernel, the bias add is fused into the output transpose
    (``sl_transpose_bias_f32``), and the output is returned contiguous, so
    the surrounding element-wise ops stay vectorised:

        forward:  X = x^T;  Y = W.X (sl_spmm_fwd);  y = Y^T (+ bias)
        backward: dY = dy^T;  dW = SDDMM(dY, X);  dX = W^T.dY (cached
                  transpose);  dx = dX^T;  dbias = dy.sum(0)

    Transposes are exact copies and the bias add is one fp32 add per element,
    so every value equals ``_SpMMFunction``'s on ``x.t()`` plus torch's bias
    add, and dbias is the reduction autograd makes for a broadcast add.
    Inputs ``(W_values, W, x, bias)`` (bias may be None); backward returns
    ``(dW_values[total_capacity], None, dx, dbias)``.
    """

    @staticmethod
    def forward(ctx, W_values, W, x, bias=None):
        if x.device.type != "cuda" or x.device != W.device:
            raise RuntimeError(f"SparseLinear: input must be on {W.device} (got {x.device}); "
                               f"sparsecore_b200 has no CPU path.")
        X = _transpose(x)
        ctx.save_for_backward(W_values, X)
        ctx.W = W
        ctx.param = W_values
        Y = _spmm_raw(W, X)
        if bias is not None and bias.dtype == torch.float32 and bias.device == Y.device:
            return _transpose_bias(Y, bias)
        y = _transpose(Y)
        return y if bias is None else y + bias

    @staticmethod
    def backward(ctx, dy):
        W_values, X = ctx.saved_tensors
        W = ctx.W
        dY = _transpose(dy)
        dW = _weight_grad(W, dY, X, ctx.param, ctx.needs_input_grad[0])
        dx = None
        if ctx.needs_input_grad[2]:
            dx = _transpose(_spmm_raw(_cached_transpose(W), dY, kind="spmm_dx"))
        db = dy.sum(0) if len(ctx.needs_input_grad) > 3 and ctx.needs_input_grad[3] else None
        return dW, None, dx, db


# ── weight gradient off the critical path ───────────────────────────────
# The SDDMM's output is consumed only by the optimizer step, while dX gates
# the rest of the backward pass.  SparseLinear therefore launches the SDDMM
# on a per-device side stream (forked from the current stream after dY is
# ready), so it overlaps the following dX / attention / transpose work, and
# joins it back at the end of the backward pass (an autograd engine
# callback, as DistributedDataParallel does): the current stream waits for
# the SDDMM and the gradient is accumulated into the Parameter's ``.grad``
# there.  Values are identical to the synchronous path.  Opt-in: with it the
# weight gradient reaches the Parameter only through ``.grad`` at the end of
# ``backward()`` -- ``torch.autograd.grad`` on the weights and hooks
# registered on the weight Parameter do not see it -- so the default keeps
# plain autograd semantics.
_async_weight_grad = False
_side_streams: dict = {}
# Callables (param, dW) run on the side stream right after a SparseLinear's
# SDDMM is enqueued there (async weight-gradient mode only); the data-
# parallel helper packs and all-reduces gradient buckets from here, so the
# exchange overlaps the rest of the backward pass.
_weight_grad_hooks: list = []


def add_weight_grad_hook(fn) -> None:
    if fn not in _weight_grad_hooks:
        _weight_grad_hooks.append(fn)


def remove_weight_grad_hook(fn) -> None:
    if fn in _weight_grad_hooks:
        _weight_grad_hooks.remove(fn)


def set_async_weight_grad(enabled: bool) -> None:
    """Run SparseLinear's weight-gradient SDDMM on a side stream, overlapped
    with the rest of the backward pass; the gradient is accumulated into the
    weight Parameter's ``.grad`` when ``backward()`` finishes (not visible to
    ``torch.autograd.grad`` or Parameter hooks).  Off by default."""
    global _async_weight_grad
    _async_weight_grad = bool(enabled)


def critical_path_stream(device=None) -> torch.cuda.Stream:
    """A highest-priority CUDA stream for running a training step.

    SparseLinear's weight-gradient SDDMM runs on a side stream of the lowest
    (default) priority; when the step itself runs on this stream, the block
    scheduler hands freed SM slots to the critical-path kernels (dX, the
    rest of the backward pass) first.  Measured on B200, config 5: 123.7 ->
    118.5 ms/step.  Use as ``torch.cuda.set_stream(critical_path_stream())``
    or ``with torch.cuda.stream(critical_path_stream()):``.
    """
    dev = N.require_cuda(device)
    _, hi = torch.cuda.Stream.priority_range()
    return torch.cuda.Stream(device=dev, priority=hi)


def _side_stream(device: torch.device) -> torch.cuda.Stream:
    s = _side_streams.get(device.index)
    if s is None:
        s = torch.cuda.Stream(device=device)
        _side_streams[device.index] = s
    return s


def _sddmm_on_side_stream(W: PaddedCSR, dY: torch.Tensor, X: torch.Tensor, param) -> None:
    main = torch.cuda.current_stream(dY.device)
    side = _side_stream(dY.device)
    side.wait_stream(main)
    with torch.cuda.stream(side):
        dW = _sddmm_raw(W, dY, X)
        for hook in _weight_grad_hooks:
            hook(param, dW)
        done = torch.cuda.Event()
        done.record(side)
    capturing = torch.cuda.is_current_stream_capturing()
    keep = (dY, X)  # alive until the join: no allocation may reuse them while the SDDMM reads

    def join():
        cur = torch.cuda.current_stream(dW.device)
        cur.wait_event(done)  # frees of `keep` after this point are ordered after the SDDMM
        if not capturing:
            dW.record_stream(cur)  # dW's block belongs to the side stream's pool
        if param.grad is None:
            param.grad = dW
        else:
            param.grad.add_(dW)
        del keep[:]

    keep = list(keep)
    torch.autograd.Variable._execution_engine.queue_callback(join)


def _weight_grad(W: PaddedCSR, dY: torch.Tensor, X: torch.Tensor, param, needed: bool):
    """dW for a SparseLinear weight: async (side stream, joined at the end of
    backward) when enabled, else returned for autograd to accumulate."""
    if not needed:
        return None
    if _async_weight_grad and param.is_leaf:
        _sddmm_on_side_stream(W, dY, X, param)
        return None
    return _sddmm_raw(W, dY, X)


class _SparseMLPFunction(torch.autograd.Function):
    """Two SparseLinears with an element-wise activation between them,
    ``y = (W2 . act(W1 . x^T + b1) + b2)^T`` (either bias may be None),
    keeping the hidden activation in the kernels' column-per-token layout:
    the transposes of the hidden tensor that two separate SparseLinear calls
    would make (one each way, forward and backward) are skipped.  b1 and the
    activation run in the first forward kernel's epilogue, b2 in the output
    transpose.  Every value equals the unfused composition: the bias adds and
    the activation and its backward are element-wise, and each bias gradient
    is the token-major reduction autograd makes for the broadcast add."""

    @staticmethod
    def forward(ctx, v1, v2, x, W1, W2, act, b1=None, b2=None):
        X = _transpose(x)
        Y1, H = _spmm_act_raw(W1, X, b1, act)
        ctx.save_for_backward(X, Y1, H)
        ctx.W1, ctx.W2, ctx.act = W1, W2, act
        ctx.p1, ctx.p2 = v1, v2
        Y2 = _spmm_raw(W2, H)
        return _transpose(Y2) if b2 is None else _transpose_bias(Y2, b2)

    @staticmethod
    def backward(ctx, dy):
        X, Y1, H = ctx.saved_tensors
        W1, W2 = ctx.W1, ctx.W2
        dY2 = _transpose(dy)
        dW2 = _weight_grad(W2, dY2, H, ctx.p2, ctx.needs_input_grad[1])
        dH = _spmm_raw(_cached_transpose(W2), dY2, kind="spmm_dx")
        if ctx.act == "gelu":
            dY1 = torch.ops.aten.gelu_backward(dH, Y1)
        else:
            dY1 = torch.ops.aten.threshold_backward(dH, H, 0)
        dW1 = _weight_grad(W1, dY1, X, ctx.p1, ctx.needs_input_grad[0])
        dx = None
        if ctx.needs_input_grad[2]:
            dx = _transpose(_spmm_raw(_cached_transpose(W1), dY1, kind="spmm_dx"))
        ng = ctx.needs_input_grad
        db1 = _transpose(dY1).sum(0) if len(ng) > 6 and ng[6] else None
        db2 = dy.sum(0) if len(ng) > 7 and ng[7] else None
        return dW1, dW2, dx, None, None, None, db1, db2


def spmm(W: PaddedCSR, X: torch.Tensor, *, kernel: str = "auto") -> torch.Tensor:
    """Y = W @ X for a PaddedCSR W (M,K) and dense CUDA X (K,N) -> (M,N) fp32.

    Routes through autograd when X or W.values requires grad.
    Raises TypeError (wrong types), ValueError (ndim / shape / kernel name),
    RuntimeError (X not on W's CUDA device).
    """
    if not isinstance(W, PaddedCSR):
        raise TypeError(f"spmm: W must be a sparselab.PaddedCSR, got {type(W).__name__}")
    if not isinstance(X, torch.Tensor):
        raise TypeError(f"spmm: X must be a torch.Tensor, got {type(X).__name__}")
    if X.device.type != "cuda":
        raise RuntimeError(f"spmm: X must be on a CUDA device (got device={X.device}). "
                           f"sparsecore_b200 has no CPU path.")
    if X.dim() != 2:
        raise ValueError(f"spmm: X must be 2-D, got shape={tuple(X.shape)}")
    if kernel not in _VALID_KERNELS:
        raise ValueError(f"spmm: unknown kernel={kernel!r}. Expected one of: "
                         f"{sorted(_VALID_KERNELS)}.")
    X_f32 = X.to(dtype=torch.float32).contiguous()
    W_values = W.values
    if X_f32.requires_grad or W_values.requires_grad:
        return _SpMMFunction.apply(W_values, W, X_f32, kernel)
    return _spmm_raw(W, _check_dense(W, X_f32, "spmm_simd"))
