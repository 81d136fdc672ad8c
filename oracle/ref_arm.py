"""CPU reference arm: the reference's own compiled kernels on the host cores.

TEST / MEASUREMENT INFRASTRUCTURE ONLY (used by bench.py's reference arm and
cpu_baseline leg).  The sparse projections call the reference's ``_core``
extension -- compiled from the reference sources by oracle/Makefile into
oracle/_ref/refcore/ -- exactly as the reference's ``_SpMMFunction`` does
(sparselab/ops.py:145-210): forward ``spmm_simd(W, X)``, backward
``spmm_grad_w_simd(W, dY, X)`` and ``spmm_simd(W^T, dY)`` over a transpose
cached per topology and value-refreshed through its permutation
(sparselab/ops.py:70-99).  Everything else (embeddings, LayerNorm, attention,
AdamW) is stock torch on the CPU, as in the reference's demos.

If the reference ``_core`` was not built, the kernels fall back to the C
oracle (single-threaded restatement) and the arm reports kind "port".
"""
from __future__ import annotations

import importlib.util
import math
import os

import numpy as np
import torch
import torch.nn as nn

from . import oracle as O

_HERE = os.path.dirname(os.path.abspath(__file__))
_core = None


def load_refcore():
    """The reference's compiled `_core` module, or None if not built."""
    global _core
    if _core is not None:
        return _core
    d = os.path.join(_HERE, "_ref", "refcore")
    if not os.path.isdir(d):
        return None
    for f in os.listdir(d):
        if f.startswith("_core") and f.endswith(".so"):
            spec = importlib.util.spec_from_file_location("_core", os.path.join(d, f))
            mod = importlib.util.module_from_spec(spec)
            spec.loader.exec_module(mod)
            _core = mod
            return mod
    return None


class _RefSpMM(torch.autograd.Function):
    @staticmethod
    def forward(ctx, W_values, layer, X):
        ctx.layer = layer
        ctx.save_for_backward(X)
        return torch.from_numpy(layer.kernels.fwd(layer.W, X.contiguous().numpy()))

    @staticmethod
    def backward(ctx, dY):
        (X,) = ctx.saved_tensors
        layer = ctx.layer
        dYn = dY.to(torch.float32).contiguous().numpy()
        dW = torch.from_numpy(layer.kernels.dw(layer.W, dYn, X.numpy()))
        WT = layer.cached_transpose()
        dX = torch.from_numpy(layer.kernels.fwd(WT, dYn))
        return dW, None, dX


class _CoreKernels:
    kind = "reference"

    def __init__(self, core):
        self.core = core

    def make(self, p: O.CSR):
        return self.core.PaddedCSR(p.nrows, p.ncols, p.values.tolist(), p.cols.tolist(),
                                   p.row_start.tolist(), p.row_nnz.tolist(),
                                   p.row_capacity.tolist())

    def values(self, W):
        return np.asarray(W.values)

    def fwd(self, W, X):
        return self.core.spmm_simd(W, X)

    def dw(self, W, dY, X):
        return self.core.spmm_grad_w_simd(W, dY, X)


class _PortKernels:
    kind = "port"

    def make(self, p: O.CSR):
        return p

    def values(self, W):
        return W.values

    def fwd(self, W, X):
        return O.spmm(W, X)

    def dw(self, W, dY, X):
        return O.sddmm(W, dY, X)


def kernels():
    core = load_refcore()
    return _CoreKernels(core) if core is not None else _PortKernels()


class RefSparseLinear(nn.Module):
    """CPU SparseLinear over the reference kernels; same init draws as the
    reference (sparselab/nn.py:118-185)."""

    def __init__(self, fin, fout, sparsity, kern, bias=False, padding_ratio=0.2):
        """bias=True adds the reference's bias (uniform +-1/sqrt(fan), drawn
        after the weights, sparselab/nn.py:113-116)."""
        super().__init__()
        self.in_features, self.out_features = fin, fout
        self.kernels = kern
        fan = max(1.0, fin * (1.0 - sparsity))
        bound = 1.0 / math.sqrt(fan)
        Wd = torch.empty(fout, fin)
        nn.init.uniform_(Wd, -bound, bound)
        mask = torch.rand(fout, fin) >= sparsity
        p = O.from_dense((Wd * mask.float()).numpy(), padding_ratio=padding_ratio)
        self._p = p
        self.W = kern.make(p)
        self._values = nn.Parameter(torch.from_numpy(kern.values(self.W)))
        self.bias = nn.Parameter(torch.empty(fout).uniform_(-bound, bound)) if bias else None
        self._wt = None

    def cached_transpose(self):
        if self._wt is None:
            # Topology is fixed inside a timed sample: build W^T once.
            pT, perm = O.transpose_with_perm(self._p)
            self._wt = (self.kernels.make(pT), perm, perm >= 0)
        WT, perm, live = self._wt
        wt_vals = self.kernels.values(WT)
        w_vals = self.kernels.values(self.W)
        wt_vals[live] = w_vals[perm[live]]
        return WT

    def forward(self, x):
        shp = x.shape
        X_col = x.reshape(-1, self.in_features).t().contiguous()
        y = _RefSpMM.apply(self._values, self, X_col).t()
        if self.bias is not None:
            y = y + self.bias
        return y.reshape(shp[:-1] + (self.out_features,))


def linear_factory(kern):
    def make(fin, fout, sparsity, bias=False):
        return RefSparseLinear(fin, fout, sparsity, kern, bias=bias)
    return make


class KernelTimer:
    """Host-core time of the reference's own kernels on the cells of one
    matrix, by the reference's timing method (examples/
    profile_phase1_timing_table.py:45-59): warm-up calls, then the median
    of 30 trials, cut to the median of 3 for calls over 1 s (and to one
    warm-up for calls over 0.2 s).  Forward ``spmm_simd(W, X)``, SDDMM
    ``spmm_grad_w_simd(W, dY, X)`` and dX ``spmm_simd(W^T, dY)`` run the
    compiled reference ``_core`` (kind "reference"); the transpose is the
    reference's Python algorithm (sparselab/layout.py:460), restated in
    numpy here (kind "port"), timed once per matrix.  Milliseconds per
    call."""

    def __init__(self, p: O.CSR):
        self.kern = kernels()
        self.p = p
        self.W = self.kern.make(p)
        pT, _ = O.transpose_with_perm(p)
        self.WT = self.kern.make(pT)
        self.transpose_ms = self._time(lambda: O.transpose_with_perm(p))

    @staticmethod
    def _time(fn):
        import statistics
        import time

        t0 = time.perf_counter()
        fn()
        first = time.perf_counter() - t0
        for _ in range(4 if first < 0.2 else 0):
            fn()
        trials = 30 if first < 1.0 else 3
        ts = []
        for _ in range(trials):
            t0 = time.perf_counter()
            fn()
            ts.append(time.perf_counter() - t0)
        return round(statistics.median(ts) * 1e3, 4)

    def cell(self, X: np.ndarray, dY: np.ndarray) -> dict:
        X = np.ascontiguousarray(X, np.float32)
        dY = np.ascontiguousarray(dY, np.float32)
        k = self.kern
        return {"fwd": self._time(lambda: k.fwd(self.W, X)),
                "dw": self._time(lambda: k.dw(self.W, dY, X)),
                "dx": self._time(lambda: k.fwd(self.WT, dY)),
                "transpose": self.transpose_ms, "kind": k.kind, "transpose_kind": "port"}


def kernel_times(p: O.CSR, X: np.ndarray, dY: np.ndarray) -> dict:
    """One cell's reference CPU times (see KernelTimer)."""
    return KernelTimer(p).cell(X, dY)
