"""CPU oracle for the padded-CSR sparse-training hot path.

TEST INFRASTRUCTURE ONLY.  Only ``tests/``, ``__graft_entry__.smoke()`` and the
CPU-baseline leg of ``bench.py`` import this module, and only as the checker
(or as the timed CPU reference arm); the product package ``sparsecore_b200``
never imports it.

Two layers:

* ``liboracle.so`` (``oracle/oracle.c``, built by ``oracle/Makefile`` into
  ``oracle/_ref/``): the numeric kernels restated in plain C with explicit
  ``fmaf`` so the rounding sequence is fixed -- forward SpMM, SDDMM dW,
  dense gradient, transpose-with-perm, invariant check.
* numpy restatements below of the Python-level algorithms of the reference
  (``sparselab/layout.py`` factories and ``sparselab/router.py`` SET/RigL
  prune-and-regrow), operating on plain numpy arrays.

All arrays follow the reference layout: ``values f32[cap]``,
``cols i32[cap]`` (padding = -1), ``row_start/row_nnz/row_capacity i32[M]``.
"""
from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_ref", "liboracle.so")
_lib = None


def lib() -> ctypes.CDLL:
    """Load (building on first use if needed) the C oracle."""
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH) or (
            os.path.getmtime(_LIB_PATH) < os.path.getmtime(os.path.join(_HERE, "oracle.c"))
        ):
            build()
        _lib = ctypes.CDLL(_LIB_PATH)
        P = ctypes.c_void_p
        I64 = ctypes.c_int64
        _lib.or_capacity.argtypes = [P, I64, ctypes.c_double, P]
        _lib.or_spmm.argtypes = [I64, I64, P, P, P, P, P, P]
        _lib.or_sddmm.argtypes = [I64, I64, I64, P, P, P, P, P, P]
        _lib.or_sddmm_sequential.argtypes = [I64, I64, I64, P, P, P, P, P, P]
        _lib.or_dense_grad.argtypes = [I64, I64, I64, P, P, P, ctypes.c_int]
        _lib.or_transpose_count.argtypes = [I64, I64, P, P, P, ctypes.c_double, P, P, P]
        _lib.or_transpose_count.restype = I64
        _lib.or_transpose_fill.argtypes = [I64, I64, P, P, P, P, P, I64, P, P, P]
        _lib.or_check_invariants.argtypes = [I64, I64, I64, P, P, P, P, P, P]
        _lib.or_check_invariants.restype = ctypes.c_int
    return _lib


def build() -> None:
    """Compile liboracle.so (and the reference `_core` when its sources exist)."""
    import subprocess

    subprocess.run(["make", "-s", "-C", _HERE, "all"], check=True)


def _p(a: np.ndarray):
    return a.ctypes.data_as(ctypes.c_void_p)


def _c(a, dtype):
    return np.ascontiguousarray(a, dtype=dtype)


@dataclass
class CSR:
    """Plain-numpy padded CSR (the reference's five arrays plus shape)."""

    nrows: int
    ncols: int
    values: np.ndarray
    cols: np.ndarray
    row_start: np.ndarray
    row_nnz: np.ndarray
    row_capacity: np.ndarray

    @property
    def nnz(self) -> int:
        return int(self.row_nnz.sum())

    @property
    def total_capacity(self) -> int:
        return int(self.row_capacity.sum())

    def copy(self) -> "CSR":
        return CSR(self.nrows, self.ncols, self.values.copy(), self.cols.copy(),
                   self.row_start.copy(), self.row_nnz.copy(), self.row_capacity.copy())


# ───────────────────────── capacity / factories ─────────────────────────

def capacity(row_nnz: np.ndarray, padding_ratio: float) -> np.ndarray:
    """sparselab/layout.py:46-68: max(1, ceil(nnz*(1+pr))) in float64."""
    if padding_ratio < 0:
        raise ValueError(f"padding_ratio must be >= 0, got {padding_ratio}")
    rn = _c(row_nnz, np.int32)
    out = np.empty_like(rn)
    lib().or_capacity(_p(rn), rn.size, 1.0 + padding_ratio, _p(out))
    return out


def from_dense(W: np.ndarray, threshold: float = 0.0, padding_ratio: float = 0.2) -> CSR:
    """sparselab/layout.py:75-208 (from_dense -> from_torch_sparse_csr):
    live = |w| > threshold when threshold > 0, else w != 0; live entries
    first in each row in ascending column order, padding (-1, 0.0)."""
    W = _c(W, np.float32)
    M, K = W.shape
    live = (np.abs(W) > threshold) if threshold > 0 else (W != 0)
    row_nnz = live.sum(axis=1).astype(np.int32)
    cap = capacity(row_nnz, padding_ratio)
    row_start = np.concatenate(([0], np.cumsum(cap[:-1]))).astype(np.int32) if M else np.zeros(0, np.int32)
    total = int(cap.sum())
    vals = np.zeros(total, np.float32)
    cols = np.full(total, -1, np.int32)
    for i in range(M):
        c = np.nonzero(live[i])[0]
        vals[row_start[i]:row_start[i] + c.size] = W[i, c]
        cols[row_start[i]:row_start[i] + c.size] = c
    return CSR(M, K, vals, cols, row_start, row_nnz, cap)


def to_dense(p: CSR) -> np.ndarray:
    """sparselab/layout.py:262-292."""
    out = np.zeros((p.nrows, p.ncols), np.float32)
    for i in range(p.nrows):
        s, n = int(p.row_start[i]), int(p.row_nnz[i])
        out[i, p.cols[s:s + n]] = p.values[s:s + n]
    return out


def check_invariants(p: CSR) -> tuple[int, int, int]:
    """csrc/kernels/padded_csr.cpp:79-196 -> (code, row, slot); code 0 = ok."""
    wr = ctypes.c_int64()
    ws = ctypes.c_int64()
    rs, rn, rc, cl = (_c(p.row_start, np.int32), _c(p.row_nnz, np.int32),
                      _c(p.row_capacity, np.int32), _c(p.cols, np.int32))
    code = lib().or_check_invariants(p.nrows, p.ncols, cl.size, _p(rs), _p(rn), _p(rc),
                                     _p(cl), ctypes.byref(wr), ctypes.byref(ws))
    return int(code), int(wr.value), int(ws.value)


# ───────────────────────────── kernels ─────────────────────────────

def spmm(p: CSR, X: np.ndarray) -> np.ndarray:
    """Y = W.X, per-element FMA chain in slot order (spmm_avx2.cpp:82-263)."""
    X = _c(X, np.float32)
    assert X.shape[0] == p.ncols
    N = X.shape[1]
    Y = np.empty((p.nrows, N), np.float32)
    rs, rn, cl, vl = (_c(p.row_start, np.int32), _c(p.row_nnz, np.int32),
                      _c(p.cols, np.int32), _c(p.values, np.float32))
    lib().or_spmm(p.nrows, N, _p(rs), _p(rn), _p(cl), _p(vl), _p(X), _p(Y))
    return Y


def sddmm(p: CSR, dY: np.ndarray, X: np.ndarray, order: str = "avx2") -> np.ndarray:
    """dW at live slots (spmm_grad_avx2.cpp:73-259), padding 0."""
    dY = _c(dY, np.float32)
    X = _c(X, np.float32)
    N = dY.shape[1]
    cap = p.total_capacity
    dW = np.empty(cap, np.float32)
    rs, rn, cl = _c(p.row_start, np.int32), _c(p.row_nnz, np.int32), _c(p.cols, np.int32)
    fn = lib().or_sddmm if order == "avx2" else lib().or_sddmm_sequential
    fn(p.nrows, N, cap, _p(rs), _p(rn), _p(cl), _p(dY), _p(X), _p(dW))
    return dW


def dense_grad(dY: np.ndarray, X: np.ndarray, order: str = "sequential") -> np.ndarray:
    """G = dY.X^T (dense_grad.cpp:463-523)."""
    dY = _c(dY, np.float32)
    X = _c(X, np.float32)
    M, N = dY.shape
    K = X.shape[0]
    G = np.empty((M, K), np.float32)
    lib().or_dense_grad(M, K, N, _p(dY), _p(X), _p(G), 1 if order == "avx2" else 0)
    return G


def transpose_with_perm(p: CSR, padding_ratio: float = 0.2) -> tuple[CSR, np.ndarray]:
    """sparselab/layout.py:460-536: (W^T, perm[slot_T] -> slot_W or -1)."""
    M, K = p.nrows, p.ncols
    rs, rn, cl, vl = (_c(p.row_start, np.int32), _c(p.row_nnz, np.int32),
                      _c(p.cols, np.int32), _c(p.values, np.float32))
    onnz = np.empty(K, np.int32)
    ocap = np.empty(K, np.int32)
    ostart = np.empty(K, np.int32)
    total = lib().or_transpose_count(M, K, _p(rs), _p(rn), _p(cl), 1.0 + padding_ratio,
                                     _p(onnz), _p(ocap), _p(ostart))
    ov = np.empty(total, np.float32)
    oc = np.empty(total, np.int32)
    perm = np.empty(total, np.int64)
    lib().or_transpose_fill(M, K, _p(rs), _p(rn), _p(cl), _p(vl), _p(ostart), total,
                            _p(ov), _p(oc), _p(perm))
    return CSR(K, M, ov, oc, ostart, onnz, ocap), perm


# ───────────────────────────── routers ─────────────────────────────

def _live_abs(p: CSR) -> np.ndarray:
    parts = [p.values[p.row_start[i]:p.row_start[i] + p.row_nnz[i]] for i in range(p.nrows)]
    return np.abs(np.concatenate(parts)) if parts else np.zeros(0, np.float32)


def drop_threshold(p: CSR, drop_fraction: float) -> np.float32:
    """sparselab/router.py:395-412: k_drop = max(1, int(df*nnz)); the k_drop-th
    smallest |v| among live slots (exact order statistic)."""
    a = _live_abs(p)
    k = max(1, int(drop_fraction * p.nnz))
    return np.partition(a, k - 1)[k - 1]


def _keep_row(live_vals: np.ndarray, thr) -> np.ndarray:
    """router.py:420-439: keep |v| > thr; none kept -> keep first argmax."""
    keep = np.abs(live_vals) > thr
    if not keep.any() and live_vals.size > 0:
        keep[int(np.argmax(np.abs(live_vals)))] = True
    return keep


def _write_row(p: CSR, i: int, new_cols: np.ndarray, new_vals: np.ndarray) -> None:
    """csrc/kernels/padded_csr.cpp:219-296 (rewrite_row) minus validation."""
    s, cap = int(p.row_start[i]), int(p.row_capacity[i])
    n = new_cols.size
    p.cols[s:s + n] = new_cols
    p.values[s:s + n] = new_vals
    p.cols[s + n:s + cap] = -1
    p.values[s + n:s + cap] = 0.0
    p.row_nnz[i] = n


def set_update(p: CSR, drop_fraction: float, rng: np.random.Generator) -> int:
    """SET global-threshold prune + random regrow on one layer, in place
    (sparselab/router.py:378-483).  Returns the number of rewritten rows
    (the reference bumps topology_version once per rewrite_row call)."""
    if p.nnz == 0:
        return 0
    thr = drop_threshold(p, drop_fraction)
    rewrites = 0
    for i in range(p.nrows):
        s, n_live = int(p.row_start[i]), int(p.row_nnz[i])
        if n_live == 0:
            continue
        lc = p.cols[s:s + n_live].copy()
        lv = p.values[s:s + n_live].copy()
        keep = _keep_row(lv, thr)
        sc, sv = lc[keep], lv[keep]
        n_drop = n_live - sc.size
        empty = np.setdiff1d(np.arange(p.ncols, dtype=np.int32), sc, assume_unique=True)
        if empty.size == 0 or n_drop == 0:
            _write_row(p, i, sc, sv)
        else:
            n_grow = min(n_drop, empty.size)
            g = rng.choice(empty, size=n_grow, replace=False).astype(np.int32)
            mc = np.concatenate([sc, g])
            mv = np.concatenate([sv, np.zeros(n_grow, np.float32)])
            o = np.argsort(mc, kind="stable")
            _write_row(p, i, mc[o], mv[o])
        rewrites += 1
    return rewrites


def rigl_update(p: CSR, drop_fraction: float, G: np.ndarray) -> int:
    """RigL prune + gradient-magnitude regrow on one layer, in place, given the
    dense gradient G[M,K] (sparselab/router.py:598-735).  Returns the number of
    rewritten rows."""
    if p.nnz == 0:
        return 0
    absG = np.abs(np.asarray(G, np.float32))
    thr = drop_threshold(p, drop_fraction)
    rewrites = 0
    for i in range(p.nrows):
        s, n_live = int(p.row_start[i]), int(p.row_nnz[i])
        if n_live == 0:
            continue
        lc = p.cols[s:s + n_live].copy()
        lv = p.values[s:s + n_live].copy()
        keep = _keep_row(lv, thr)
        sc, sv = lc[keep], lv[keep]
        n_drop = n_live - sc.size
        rewrites += 1
        if n_drop == 0:
            _write_row(p, i, sc, sv)
            continue
        row = absG[i].copy()
        row[sc] = -np.inf
        avail = int((row > -np.inf).sum())
        n_grow = min(n_drop, avail)
        if n_grow == 0:
            _write_row(p, i, sc, sv)
            continue
        g = np.argpartition(-row, n_grow - 1)[:n_grow].astype(np.int32)
        mc = np.concatenate([sc, g])
        mv = np.concatenate([sv, np.zeros(n_grow, np.float32)])
        o = np.argsort(mc, kind="stable")
        _write_row(p, i, mc[o], mv[o])
    return rewrites
