"""Device-resident padded CSR and its factories.

Mirrors the reference's storage type and Python factories:

* ``PaddedCSR`` -- ``csrc/kernels/padded_csr.hpp:47-143`` and its Python
  surface ``csrc/bindings.cpp:599-744`` (constructors, properties,
  ``assert_invariants``, ``rewrite_row``, ``__repr__``);
* ``from_dense`` / ``from_torch_sparse_csr`` / ``random`` / ``to_dense`` /
  ``transpose`` / ``transpose_with_perm`` -- ``sparselab/layout.py:75-536``.

The five arrays live in CUDA memory as torch tensors (``values`` float32,
the rest int32); small host mirrors of the per-row arrays keep ``nnz``,
capacities and validation free of device round trips.  ``values`` is the
tensor a ``SparseLinear`` parameter aliases; structural arrays are meant to be
read-only (mutate topology only through ``rewrite_row`` or a router).
All computation runs in the sparsecore_b200 CUDA library.
"""
from __future__ import annotations

import ctypes

import numpy as np
import torch

from . import _native as N

__all__ = [
    "PaddedCSR",
    "from_dense",
    "from_torch_sparse_csr",
    "random",
    "to_dense",
    "transpose",
    "transpose_with_perm",
]


def _to_host_i32(a, name: str) -> np.ndarray:
    if isinstance(a, torch.Tensor):
        a = a.detach().cpu().numpy()
    arr = np.asarray(a)
    if arr.ndim != 1:
        raise ValueError(f"PaddedCSR: {name} must be 1-D")
    return np.ascontiguousarray(arr, dtype=np.int32)


def _to_dev(a, dtype: torch.dtype, device: torch.device) -> torch.Tensor:
    if isinstance(a, torch.Tensor):
        return a.detach().to(device=device, dtype=dtype).contiguous().clone()
    return torch.as_tensor(np.asarray(a), dtype=dtype).to(device).contiguous()


class PaddedCSR:
    """Padded-row CSR sparse matrix in CUDA memory.

    ``PaddedCSR(nrows, ncols)`` builds an empty (zero-capacity) matrix;
    ``PaddedCSR(nrows, ncols, values, col_indices, row_start, row_nnz,
    row_capacity)`` takes the five arrays (lists, numpy arrays or tensors)
    and validates all invariants, raising ``ValueError`` on violation
    (``csrc/bindings.cpp:604-627``).
    """

    def __init__(self, nrows: int, ncols: int, values=None, col_indices=None, row_start=None,
                 row_nnz=None, row_capacity=None, *, device=None):
        dev = N.require_cuda(device)
        nrows, ncols = int(nrows), int(ncols)
        if nrows < 0 or ncols < 0:
            raise ValueError(
                f"PaddedCSR invariant check failed: Invariant 1 violated: shape must be "
                f"non-negative, got ({nrows}, {ncols}).")
        full = [values, col_indices, row_start, row_nnz, row_capacity]
        if all(a is None for a in full):
            z = np.zeros(nrows, np.int32)
            self._init_arrays(nrows, ncols, torch.zeros(0, dtype=torch.float32, device=dev),
                              torch.zeros(0, dtype=torch.int32, device=dev), z, z.copy(), z.copy(), dev)
            return
        if any(a is None for a in full):
            raise TypeError("PaddedCSR: give either (nrows, ncols) or all five arrays")
        rs, rn, rc = (_to_host_i32(row_start, "row_start"), _to_host_i32(row_nnz, "row_nnz"),
                      _to_host_i32(row_capacity, "row_capacity"))
        vals = _to_dev(values, torch.float32, dev).reshape(-1)
        cols = _to_dev(col_indices, torch.int32, dev).reshape(-1)
        self._init_arrays(nrows, ncols, vals, cols, rs, rn, rc, dev)
        self.assert_invariants()

    # ── construction helpers ────────────────────────────────────────────
    def _init_arrays(self, nrows, ncols, vals, cols, rs_h, rn_h, rc_h, dev, rs_d=None, rn_d=None,
                     rc_d=None):
        self._nrows, self._ncols, self._device = nrows, ncols, dev
        self._values, self._cols = vals, cols
        self._rs_h, self._rn_h, self._rc_h = rs_h, rn_h, rc_h
        self._row_start = rs_d if rs_d is not None else torch.from_numpy(rs_h.copy()).to(dev)
        self._row_nnz = rn_d if rn_d is not None else torch.from_numpy(rn_h.copy()).to(dev)
        self._row_capacity = rc_d if rc_d is not None else torch.from_numpy(rc_h.copy()).to(dev)
        self._nnz = int(rn_h.astype(np.int64).sum())
        self.topology_version_ = 0
        self._abi = None

    @classmethod
    def _from_device(cls, nrows, ncols, vals, cols, rs_d, rn_d, rc_d, dev) -> "PaddedCSR":
        """Wrap arrays produced by our own kernels (already valid)."""
        obj = cls.__new__(cls)
        host = torch.stack([rs_d, rn_d, rc_d]).cpu().numpy() if nrows else np.zeros((3, 0), np.int32)
        obj._init_arrays(nrows, ncols, vals, cols, host[0].copy(), host[1].copy(), host[2].copy(),
                         dev, rs_d, rn_d, rc_d)
        return obj

    def _sync_row_nnz_from_device(self) -> None:
        """Refresh the host mirrors after a device-side topology rewrite."""
        self._rn_h = self._row_nnz.cpu().numpy().copy()
        self._nnz = int(self._rn_h.astype(np.int64).sum())

    # ── C-ABI view ──────────────────────────────────────────────────────
    def _abi_ref(self):
        if self._abi is None:
            self._abi = N.SlCsr(self._nrows, self._ncols, int(self._values.numel()),
                                self._values.data_ptr(), self._cols.data_ptr(),
                                self._row_start.data_ptr(), self._row_nnz.data_ptr(),
                                self._row_capacity.data_ptr())
        return ctypes.byref(self._abi)

    def _stream(self):
        return N.stream_ptr(self._device)

    # ── properties (csrc/bindings.cpp:630-682) ──────────────────────────
    @property
    def shape(self) -> tuple[int, int]:
        return (self._nrows, self._ncols)

    @property
    def nrows(self) -> int:
        return self._nrows

    @property
    def ncols(self) -> int:
        return self._ncols

    @property
    def device(self) -> torch.device:
        return self._device

    @property
    def nnz(self) -> int:
        return self._nnz

    @property
    def total_capacity(self) -> int:
        return int(self._values.numel())

    @property
    def padding_slots(self) -> int:
        return self.total_capacity - self._nnz

    @property
    def sparsity(self) -> float:
        if self._nrows == 0 or self._ncols == 0:
            return 1.0
        return 1.0 - self._nnz / float(self._nrows * self._ncols)

    @property
    def topology_version(self) -> int:
        return self.topology_version_

    @property
    def values(self) -> torch.Tensor:
        return self._values

    @property
    def col_indices(self) -> torch.Tensor:
        return self._cols

    @property
    def row_start(self) -> torch.Tensor:
        return self._row_start

    @property
    def row_nnz(self) -> torch.Tensor:
        return self._row_nnz

    @property
    def row_capacity(self) -> torch.Tensor:
        return self._row_capacity

    def __repr__(self) -> str:
        return (f"PaddedCSR(nrows={self._nrows}, ncols={self._ncols}, nnz={self._nnz}, "
                f"capacity={self.total_capacity})")

    # ── invariants (csrc/kernels/padded_csr.cpp:79-203) ─────────────────
    def check_invariants_str(self) -> str:
        rs, rn, rc = self._rs_h, self._rn_h, self._rc_h
        M = self._nrows
        if len(rs) != M or len(rn) != M or len(rc) != M:
            return (f"Metadata array length mismatch: row_start={len(rs)}, row_nnz={len(rn)}, "
                    f"row_capacity={len(rc)}, expected nrows={M}.")
        nv, nc = int(self._values.numel()), int(self._cols.numel())
        if nv != nc:
            return (f"Invariant 2 violated: values ({nv}) and col_indices ({nc}) must have "
                    f"the same length.")
        total = int(rc.astype(np.int64).sum())
        if nv != total:
            return (f"Invariant 2 violated: values.size()={nv} does not match "
                    f"total_capacity={total} (sum of row_capacity).")
        rep = torch.empty(4, dtype=torch.int64, device=self._device)
        N.call("sl_check_invariants", self._abi_ref(), nv, N.ptr(rep), self._stream())
        code, row, slot, _ = (int(v) for v in rep.cpu().tolist())
        if code == 0:
            return ""
        if code == 3:
            if row == 0:
                return f"Invariant 3 violated: row_start[0] must be 0, got {int(rs[0])}."
            exp = int(rs[row - 1]) + int(rc[row - 1])
            return (f"Invariant 3 violated: row_start[{row}]={int(rs[row])} should equal "
                    f"row_start[{row - 1}] + row_capacity[{row - 1}] = {exp}.")
        if code == 4:
            return (f"Invariant 4 violated at row {row}: row_nnz={int(rn[row])} must be in "
                    f"[0, {int(rc[row])}].")
        c = int(self._cols[int(rs[row]) + slot].item())
        if code == 6:
            if c < 0 or c >= self._ncols:
                return (f"Invariant 6 violated at row {row}, slot {slot}: col_indices={c} "
                        f"must be in [0, {self._ncols}).")
            prev = int(self._cols[int(rs[row]) + slot - 1].item()) if slot > 0 else -1
            return (f"Invariant 6 violated at row {row}, slot {slot}: col_indices={c} must be "
                    f"strictly greater than previous={prev} (live columns must be sorted "
                    f"ascending and distinct).")
        return (f"Invariants 5+7 violated at row {row}, slot {slot}: padding col_indices={c} "
                f"must be -1.")

    def assert_invariants(self) -> None:
        err = self.check_invariants_str()
        if err:
            raise ValueError("PaddedCSR invariant check failed: " + err)

    # ── mutation (csrc/kernels/padded_csr.cpp:219-296) ──────────────────
    def rewrite_row(self, row_idx: int, new_cols, new_values) -> None:
        cols = np.asarray(new_cols.detach().cpu() if isinstance(new_cols, torch.Tensor) else new_cols)
        vals = np.asarray(new_values.detach().cpu() if isinstance(new_values, torch.Tensor) else new_values)
        if cols.ndim != 1 or vals.ndim != 1:
            raise ValueError("rewrite_row: new_cols and new_values must be 1-D arrays")
        cols = np.ascontiguousarray(cols, dtype=np.int32)
        vals = np.ascontiguousarray(vals, dtype=np.float32)
        row_idx = int(row_idx)
        if row_idx < 0 or row_idx >= self._nrows:
            raise ValueError(f"rewrite_row: row_idx={row_idx} out of range [0, {self._nrows}).")
        if cols.size != vals.size:
            raise ValueError(f"rewrite_row: new_cols.size()={cols.size} must equal "
                             f"new_values.size()={vals.size}")
        cap = int(self._rc_h[row_idx])
        n = int(cols.size)
        if n > cap:
            raise ValueError(f"rewrite_row: row {row_idx} has capacity {cap} but got {n} new "
                             f"entries.")
        prev = -1
        for k in range(n):
            c = int(cols[k])
            if c < 0 or c >= self._ncols:
                raise ValueError(f"rewrite_row: new_cols[{k}]={c} out of range [0, "
                                 f"{self._ncols}).")
            if c <= prev:
                raise ValueError(f"rewrite_row: new_cols must be strictly ascending, got {prev} "
                                 f"followed by {c} at position {k}.")
            prev = c
        base = int(self._rs_h[row_idx])
        row_c = np.full(cap, -1, np.int32)
        row_v = np.zeros(cap, np.float32)
        row_c[:n] = cols
        row_v[:n] = vals
        self._cols[base:base + cap].copy_(torch.from_numpy(row_c))
        self._values[base:base + cap].copy_(torch.from_numpy(row_v))
        self._row_nnz[row_idx] = n
        self._nnz += n - int(self._rn_h[row_idx])
        self._rn_h[row_idx] = n
        self.topology_version_ += 1

    # ── factories attached as on the reference class (__init__.py:56-64) ─
    @staticmethod
    def from_dense(W, *, threshold: float = 0.0, padding_ratio: float = 0.2, device=None):
        return from_dense(W, threshold=threshold, padding_ratio=padding_ratio, device=device)

    @staticmethod
    def from_torch_sparse_csr(csr, *, padding_ratio: float = 0.2, device=None):
        return from_torch_sparse_csr(csr, padding_ratio=padding_ratio, device=device)

    @staticmethod
    def random(nrows, ncols, *, sparsity, padding_ratio: float = 0.2, seed=None, device=None):
        return random(nrows, ncols, sparsity=sparsity, padding_ratio=padding_ratio, seed=seed,
                      device=device)

    def to_dense(self) -> torch.Tensor:
        return to_dense(self)

    def transpose(self, *, padding_ratio: float = 0.2) -> "PaddedCSR":
        return transpose(self, padding_ratio=padding_ratio)


# ─────────────────────────────── factories ───────────────────────────────

def _check_padding_ratio(padding_ratio: float) -> float:
    if padding_ratio < 0:
        raise ValueError(f"padding_ratio must be >= 0, got {padding_ratio}")
    return 1.0 + float(padding_ratio)


def _alloc_rows(M: int, dev: torch.device):
    return (torch.empty(M, dtype=torch.int32, device=dev), torch.empty(M, dtype=torch.int32, device=dev),
            torch.empty(M, dtype=torch.int32, device=dev), torch.empty(1, dtype=torch.int64, device=dev))


def from_dense(W: torch.Tensor, *, threshold: float = 0.0, padding_ratio: float = 0.2,
               device=None) -> PaddedCSR:
    """Dense 2-D tensor -> PaddedCSR (sparselab/layout.py:172-208).

    Live entries: ``|w| > threshold`` when threshold > 0, else ``w != 0``.
    A CPU ``W`` is copied to ``device`` (default: current CUDA device).
    """
    if W.dim() != 2:
        raise ValueError(f"from_dense expected 2-D tensor, got {W.dim()}-D")
    opp = _check_padding_ratio(padding_ratio)
    dev = N.require_cuda(device if device is not None else (W.device if W.is_cuda else None))
    D = W.detach().to(device=dev, dtype=torch.float32).contiguous()
    M, K = D.shape
    row_nnz, row_cap, row_start, total = _alloc_rows(M, dev)
    s = N.stream_ptr(dev)
    N.call("sl_dense_count", N.ptr(D), M, K, float(threshold), opp, N.ptr(row_nnz),
                                   N.ptr(row_cap), N.ptr(row_start), N.ptr(total), s)
    cap = int(total.item())
    vals = torch.empty(cap, dtype=torch.float32, device=dev)
    cols = torch.empty(cap, dtype=torch.int32, device=dev)
    out = PaddedCSR._from_device(M, K, vals, cols, row_start, row_nnz, row_cap, dev)
    N.call("sl_dense_fill", N.ptr(D), float(threshold), out._abi_ref(), s)
    return out


def from_torch_sparse_csr(csr: torch.Tensor, *, padding_ratio: float = 0.2,
                          device=None) -> PaddedCSR:
    """torch sparse CSR tensor -> PaddedCSR (sparselab/layout.py:75-165)."""
    if csr.layout != torch.sparse_csr:
        raise ValueError(f"from_torch_sparse_csr expected layout=torch.sparse_csr, "
                         f"got layout={csr.layout}")
    if csr.dim() != 2:
        raise ValueError(f"from_torch_sparse_csr expected 2-D tensor, got {csr.dim()}-D")
    opp = _check_padding_ratio(padding_ratio)
    dev = N.require_cuda(device if device is not None else (csr.device if csr.is_cuda else None))
    M, K = csr.size()
    crow = csr.crow_indices().to(device=dev, dtype=torch.int64).contiguous()
    tcol = csr.col_indices().to(device=dev, dtype=torch.int32).contiguous()
    tval = csr.values().to(device=dev, dtype=torch.float32).contiguous()
    row_nnz = (crow[1:] - crow[:-1]).to(torch.int32).contiguous()
    _, row_cap, row_start, total = _alloc_rows(M, dev)
    N.call("sl_capacity_scan", N.ptr(row_nnz), M, opp, N.ptr(row_cap), N.ptr(row_start),
                                     N.ptr(total), N.stream_ptr(dev))
    cap = int(total.item())
    vals = torch.zeros(cap, dtype=torch.float32, device=dev)
    cols = torch.full((cap,), -1, dtype=torch.int32, device=dev)
    nnz = int(tcol.numel())
    if nnz:
        row_of = torch.repeat_interleave(torch.arange(M, device=dev), row_nnz.long(),
                                         output_size=nnz)
        dst = row_start.long()[row_of] + (torch.arange(nnz, device=dev) - crow[:-1][row_of])
        vals[dst] = tval
        cols[dst] = tcol
    return PaddedCSR._from_device(int(M), int(K), vals, cols, row_start, row_nnz, row_cap, dev)


def random(nrows: int, ncols: int, *, sparsity: float, padding_ratio: float = 0.2,
           seed: int | None = None, device=None) -> PaddedCSR:
    """Random pattern with N(0,1) values (sparselab/layout.py:215-255).

    Draws from a CPU ``torch.Generator`` exactly as the reference does (randn,
    then rand < density), so the same seed yields the same matrix.
    """
    if not 0.0 <= sparsity < 1.0:
        raise ValueError(f"sparsity must be in [0, 1), got {sparsity}")
    gen = torch.Generator()
    if seed is not None:
        gen.manual_seed(seed)
    density = 1.0 - sparsity
    W = torch.randn(nrows, ncols, generator=gen, dtype=torch.float32)
    keep = torch.rand(nrows, ncols, generator=gen) < density
    W = W * keep.float()
    return from_dense(W, threshold=0.0, padding_ratio=padding_ratio, device=device)


def to_dense(p: PaddedCSR) -> torch.Tensor:
    """PaddedCSR -> dense float32 CUDA tensor (sparselab/layout.py:262-292)."""
    out = torch.empty(p.nrows, p.ncols, dtype=torch.float32, device=p.device)
    N.call("sl_to_dense", p._abi_ref(), N.ptr(out), p._stream())
    return out


def transpose_with_perm(p: PaddedCSR, *, padding_ratio: float = 0.2):
    """(W^T, perm) as sparselab/layout.py:460-536: output row k lists source
    rows ascending; perm[slot_T] = source slot (int64), -1 for padding."""
    opp = _check_padding_ratio(padding_ratio)
    dev = p.device
    M, K = p.nrows, p.ncols
    lib = N.lib()
    s = p._stream()
    row_nnz, row_cap, row_start, total = _alloc_rows(K, dev)
    scratch = torch.empty(int(lib.sl_transpose_scratch_bytes(M, K)), dtype=torch.uint8, device=dev)
    N.call("sl_transpose_count", p._abi_ref(), opp, N.ptr(row_nnz), N.ptr(row_cap),
                                   N.ptr(row_start), N.ptr(total), N.ptr(scratch), s)
    capT = int(total.item())
    vals = torch.empty(capT, dtype=torch.float32, device=dev)
    cols = torch.empty(capT, dtype=torch.int32, device=dev)
    perm = torch.empty(capT, dtype=torch.int64, device=dev)
    WT = PaddedCSR._from_device(K, M, vals, cols, row_start, row_nnz, row_cap, dev)
    N.call("sl_transpose_fill", p._abi_ref(), WT._abi_ref(), N.ptr(perm), N.ptr(scratch), s)
    return WT, perm


def transpose(p: PaddedCSR, *, padding_ratio: float = 0.2) -> PaddedCSR:
    """W^T as a new PaddedCSR (sparselab/layout.py:307-434)."""
    return transpose_with_perm(p, padding_ratio=padding_ratio)[0]
