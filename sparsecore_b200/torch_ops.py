"""The library's compute entry points registered as torch operators.

``torch.ops.sparselab.spmm_fwd`` and ``torch.ops.sparselab.sddmm_dw`` take a
padded CSR as its five device arrays (the layout of ``sparselab.PaddedCSR``:
values, col_indices, row_start, row_nnz, row_capacity) plus the column
count, and call the same kernels as ``ops.spmm`` (``sl_spmm_fwd``,
``sl_sddmm_dw``) on the current CUDA stream.  They replace the reference's
``_core.spmm_simd`` and ``_core.spmm_grad_w_simd`` bindings
(``csrc/bindings.cpp:253``, ``sparselab/ops.py:164,191``) for callers that
want torch operators (dispatcher, fake-tensor shape propagation) rather than
the ctypes calls; dX is ``spmm_fwd`` on the transposed CSR, as in the
reference (``sparselab/ops.py:201-203``).

The operators are registered for CUDA only, with fake (meta) implementations
for shape inference; a CPU tensor raises, as there is no CPU path.  They carry
no autograd formula of their own: the differentiable entry point stays
``sparselab.spmm`` / ``ops._SpMMFunction``.
"""
from __future__ import annotations

import ctypes

import torch

from . import _native as N

__all__ = ["spmm_fwd", "sddmm_dw"]


def _csr(values, col_indices, row_start, row_nnz, row_capacity, ncols):
    for name, t, dt in (("values", values, torch.float32), ("col_indices", col_indices, torch.int32),
                        ("row_start", row_start, torch.int32), ("row_nnz", row_nnz, torch.int32),
                        ("row_capacity", row_capacity, torch.int32)):
        if t.dtype != dt or not t.is_contiguous() or t.dim() != 1:
            raise ValueError(f"sparselab ops: {name} must be a contiguous 1-D {dt} tensor")
    return N.SlCsr(row_start.numel(), int(ncols), values.numel(), values.data_ptr(),
                   col_indices.data_ptr(), row_start.data_ptr(), row_nnz.data_ptr(),
                   row_capacity.data_ptr())


@torch.library.custom_op("sparselab::spmm_fwd", mutates_args=(), device_types="cuda")
def spmm_fwd(values: torch.Tensor, col_indices: torch.Tensor, row_start: torch.Tensor,
             row_nnz: torch.Tensor, row_capacity: torch.Tensor, ncols: int,
             X: torch.Tensor) -> torch.Tensor:
    """Y[nrows, N] = W . X for W given by its padded-CSR arrays (W is nrows x ncols)."""
    csr = _csr(values, col_indices, row_start, row_nnz, row_capacity, ncols)
    X = X.to(torch.float32).contiguous()
    if X.dim() != 2:
        raise ValueError(f"spmm_fwd: X must be 2-D, got {X.dim()}-D")
    Y = torch.empty(row_start.numel(), X.shape[1], dtype=torch.float32, device=X.device)
    N.call("sl_spmm_fwd", ctypes.byref(csr), N.ptr(X), X.shape[0], X.shape[1], N.ptr(Y),
           N.stream_ptr(X.device))
    return Y


@spmm_fwd.register_fake
def _spmm_fwd_fake(values, col_indices, row_start, row_nnz, row_capacity, ncols, X):
    return X.new_empty(row_start.shape[0], X.shape[1], dtype=torch.float32)


@torch.library.custom_op("sparselab::sddmm_dw", mutates_args=(), device_types="cuda")
def sddmm_dw(values: torch.Tensor, col_indices: torch.Tensor, row_start: torch.Tensor,
             row_nnz: torch.Tensor, row_capacity: torch.Tensor, ncols: int, dY: torch.Tensor,
             X: torch.Tensor) -> torch.Tensor:
    """dW[total_capacity]: (dY . X^T) at W's live slots, padding slots 0."""
    csr = _csr(values, col_indices, row_start, row_nnz, row_capacity, ncols)
    dY = dY.to(torch.float32).contiguous()
    X = X.to(torch.float32).contiguous()
    dW = torch.empty(values.numel(), dtype=torch.float32, device=dY.device)
    N.call("sl_sddmm_dw", ctypes.byref(csr), N.ptr(dY), N.ptr(X), dY.shape[1], N.ptr(dW),
           N.stream_ptr(dY.device))
    return dW


@sddmm_dw.register_fake
def _sddmm_dw_fake(values, col_indices, row_start, row_nnz, row_capacity, ncols, dY, X):
    return values.new_empty(values.shape[0], dtype=torch.float32)
