"""Pluggable dynamic-sparsity algorithms (mirrors sparselab/router.py).

``SparsityAlgorithm`` / ``Static`` / ``DynamicSparsityAlgorithm`` keep the
reference's attach / ``model.apply(algo)`` / ``step()`` / ``update()``
contract (router.py:61-289).  ``SET`` (router.py:296-483) and ``RigL``
(router.py:490-735) compute the same new topology as the reference, but the
prune / regrow rewrite runs on the GPU:

1. ``sl_dst_threshold`` -- exact k-th smallest |v| over the layer's live
   slots (k = max(1, int(drop_fraction * nnz))), radix select on device;
2. ``sl_dst_keep`` -- per-row survivor counts with the reference's
   force-keep of the first max-|v| slot;
3. SET: the host replays the reference's random draws -- for each row with
   live slots, drops and free columns, in row order,
   ``rng.choice(pool, n_grow, replace=False)`` on the algorithm's own
   ``numpy.random.default_rng(seed)`` (``Generator.choice(arr, n)`` equals
   ``arr[Generator.choice(len(arr), n)]`` draw for draw) -- and
   ``sl_dst_apply_random`` maps the ranks onto the row's free columns and
   rewrites every live row in place;
   RigL: ``sl_dense_grad`` gives G = dY.X^T from the captured X / dY, and
   ``sl_dst_apply_topk`` grows the largest-|G| free columns; rows whose
   choice is not unique (ties at the cut) are resolved on the host exactly
   as the reference does (``np.argpartition``) and written with
   ``sl_dst_apply_cols``.

``topology_version`` advances by the number of rewritten rows, as the
reference's per-row ``rewrite_row`` calls do.
"""
from __future__ import annotations

from typing import TYPE_CHECKING

import ctypes

import numpy as np
import torch

from . import _native as N

if TYPE_CHECKING:
    from .nn import SparseLinear

__all__ = ["SparsityAlgorithm", "DynamicSparsityAlgorithm", "Static", "SET", "RigL"]


class SparsityAlgorithm:
    """Base class for sparsity policies attached to SparseLinear layers."""

    def __init__(self, sparsity: float):
        if not (0.0 <= sparsity < 1.0):
            raise ValueError(f"sparsity must be in [0.0, 1.0), got {sparsity}")
        self.sparsity = sparsity
        self.layers: list["SparseLinear"] = []
        self._step_idx: int = 0

    def attach(self, layer: "SparseLinear") -> None:
        from .nn import SparseLinear

        if not isinstance(layer, SparseLinear):
            raise TypeError(f"SparsityAlgorithm.attach expects a SparseLinear, got "
                            f"{type(layer).__name__}")
        if layer not in self.layers:
            self.layers.append(layer)
            layer._sparsity_algorithm = self

    def __call__(self, module) -> None:
        from .nn import SparseLinear

        if isinstance(module, SparseLinear):
            self.attach(module)

    def step(self) -> None:
        self._step_idx += 1

    def update(self) -> None:  # pragma: no cover - abstract
        raise NotImplementedError("SparsityAlgorithm.update() must be overridden by subclasses")

    def __repr__(self) -> str:
        return (f"{type(self).__name__}(sparsity={self.sparsity}, n_layers={len(self.layers)}, "
                f"step={self._step_idx})")


class Static(SparsityAlgorithm):
    """Keeps the init-time mask for the whole run (router.py:184-215)."""

    def update(self) -> None:
        pass


class DynamicSparsityAlgorithm(SparsityAlgorithm):
    """Base for algorithms that mutate topology every ``update_freq`` steps."""

    def __init__(self, sparsity: float, drop_fraction: float, update_freq: int):
        super().__init__(sparsity=sparsity)
        if not (0.0 < drop_fraction <= 1.0):
            raise ValueError(f"drop_fraction must be in (0.0, 1.0], got {drop_fraction}")
        if update_freq < 1:
            raise ValueError(f"update_freq must be >= 1, got {update_freq}")
        self.drop_fraction = drop_fraction
        self.update_freq = update_freq
        # Step index of the last update() triggered by step(); the data-
        # parallel helper uses it to know when to broadcast the topology.
        self.last_update_step: int | None = None

    def step(self) -> None:
        self._step_idx += 1
        if self._step_idx % self.update_freq == 0:
            # The update reads values and gradients the kernels produced, and
            # synchronises anyway: first make sure no bounded device wait
            # gave up since the last check (its outputs would be incomplete).
            for dev in {m._csr.values.device for m in self.layers}:
                N.check_device_status(dev)
            self.update()
            self.last_update_step = self._step_idx

    def __repr__(self) -> str:
        return (f"{type(self).__name__}(sparsity={self.sparsity}, "
                f"drop_fraction={self.drop_fraction}, update_freq={self.update_freq}, "
                f"n_layers={len(self.layers)}, step={self._step_idx})")


# ───────────────────────────── shared GPU prune ─────────────────────────────

class _Prune:
    """Device threshold + survivor counts for one layer."""

    def __init__(self, csr, drop_fraction: float):
        dev = csr.device
        self.csr = csr
        lib = N.lib()
        s = csr._stream()
        total = csr.nnz
        self.k_drop = max(1, int(drop_fraction * total))
        self.thr = torch.empty(1, dtype=torch.float32, device=dev)
        scratch = torch.empty(int(lib.sl_dst_scratch_bytes()), dtype=torch.uint8, device=dev)
        N.call("sl_dst_threshold", csr._abi_ref(), self.k_drop, N.ptr(self.thr), N.ptr(scratch), s)
        self.n_keep = torch.empty(csr.nrows, dtype=torch.int32, device=dev)
        self.force = torch.empty(csr.nrows, dtype=torch.int32, device=dev)
        N.call("sl_dst_keep", csr._abi_ref(), N.ptr(self.thr), N.ptr(self.n_keep),
                                N.ptr(self.force), s)

    def finish(self) -> int:
        """Refresh host mirrors; bump the version per rewritten (live) row."""
        csr = self.csr
        live_rows = int((csr._rn_h > 0).sum())
        csr._sync_row_nnz_from_device()
        csr.topology_version_ += live_rows
        return live_rows


def _check_cols(csr) -> None:
    if csr.ncols > int(N.lib().sl_dst_max_ncols()):
        raise RuntimeError(f"router: ncols={csr.ncols} exceeds the rewrite kernel's maximum "
                           f"of {int(N.lib().sl_dst_max_ncols())}")


def _regrow_draws(rng: np.random.Generator, n_live: np.ndarray, n_keep: np.ndarray,
                  ncols: int) -> tuple[np.ndarray, np.ndarray]:
    """Per-row SET regrow ranks, as the reference's loop of
    ``rng.choice(pool, size=n_grow, replace=False)`` over the live rows
    (sparselab/router.py:457-470) draws them, and with ``rng`` advanced to
    the same state afterwards.  A PCG64 generator (``default_rng``) runs in
    ``sl_set_regrow_draws``; any other bit generator takes the per-row loop.
    Returns (counts[int32, nrows], ranks[int32, sum(counts)])."""
    n_live = np.ascontiguousarray(n_live, dtype=np.int32)
    n_keep = np.ascontiguousarray(n_keep, dtype=np.int32)
    nrows = n_live.shape[0]
    st = rng.bit_generator.state
    if st.get("bit_generator") != "PCG64":
        counts = np.zeros(nrows, np.int32)
        draws = []
        for i in np.nonzero(n_live)[0]:
            nk = int(n_keep[i])
            n_drop, pool = int(n_live[i]) - nk, ncols - nk
            if pool == 0 or n_drop == 0:
                continue
            n_grow = min(n_drop, pool)
            draws.append(rng.choice(pool, size=n_grow, replace=False))
            counts[i] = n_grow
        ranks = np.concatenate(draws).astype(np.int32) if draws else np.zeros(0, np.int32)
        return counts, ranks
    m64 = (1 << 64) - 1
    s128, inc = int(st["state"]["state"]), int(st["state"]["inc"])
    pcg = np.array([s128 >> 64, s128 & m64, inc >> 64, inc & m64], dtype=np.uint64)
    has32 = np.array([int(st["has_uint32"])], dtype=np.int32)
    u32 = np.array([int(st["uinteger"])], dtype=np.uint32)
    counts = np.zeros(nrows, np.int32)
    cap = int(np.maximum(n_live.astype(np.int64) - n_keep, 0).sum())
    ranks = np.zeros(max(cap, 1), np.int32)
    n_ranks = np.zeros(1, np.int64)
    c = ctypes
    N.call("sl_set_regrow_draws", pcg.ctypes.data_as(c.c_void_p), has32.ctypes.data_as(c.c_void_p),
           u32.ctypes.data_as(c.c_void_p), nrows, n_live.ctypes.data_as(c.c_void_p),
           n_keep.ctypes.data_as(c.c_void_p), ncols, counts.ctypes.data_as(c.c_void_p),
           ranks.ctypes.data_as(c.c_void_p), cap, n_ranks.ctypes.data_as(c.c_void_p))
    st["state"]["state"] = (int(pcg[0]) << 64) | int(pcg[1])
    st["has_uint32"] = int(has32[0])
    st["uinteger"] = int(u32[0])
    rng.bit_generator.state = st
    return counts, ranks[: int(n_ranks[0])]


class SET(DynamicSparsityAlgorithm):
    """Sparse Evolutionary Training (Mocanu et al. 2018): global magnitude
    prune, random regrow at zero (router.py:296-483)."""

    def __init__(self, sparsity: float, drop_fraction: float = 0.3, update_freq: int = 100,
                 seed: int | None = None):
        super().__init__(sparsity=sparsity, drop_fraction=drop_fraction, update_freq=update_freq)
        self._rng = np.random.default_rng(seed)

    def update(self) -> None:
        for layer in self.layers:
            self._update_layer(layer, self._rng)

    def _update_layer(self, layer, rng) -> None:
        csr = layer._csr
        if csr.nnz == 0:
            return
        _check_cols(csr)
        pr = _Prune(csr, self.drop_fraction)
        counts, ranks = _regrow_draws(rng, csr._rn_h, pr.n_keep.cpu().numpy(), csr.ncols)
        off = np.zeros(csr.nrows + 1, np.int32)
        np.cumsum(counts, out=off[1:])
        if ranks.size == 0:
            ranks = np.zeros(1, np.int32)
        dev = csr.device
        off_d = torch.from_numpy(off).to(dev)
        ranks_d = torch.from_numpy(ranks).to(dev)
        N.call("sl_dst_apply_random", csr._abi_ref(), N.ptr(pr.thr), N.ptr(pr.force),
                                            N.ptr(off_d), N.ptr(ranks_d), csr._stream())
        pr.finish()


class RigL(DynamicSparsityAlgorithm):
    """Rigging the Lottery (Evci et al. 2020): global magnitude prune, regrow
    at the largest dense-gradient magnitudes (router.py:490-735).

    ``capture="every_step"`` (default, the reference's behaviour) clones each
    layer's input and output gradient on every step; ``capture="update_step"``
    clones them only on steps whose ``step()`` will trigger an update.

    ``fused_grow=True`` (default) picks the grown columns without
    materialising the M x K dense gradient: the gradient GEMM keeps each
    row's best candidates per 128-column tile and a merge kernel selects the
    row's top n_grow (``sl_rigl_prep / sl_rigl_candidates / sl_rigl_merge``).
    Rows whose cut is a tie (or holds a NaN) are resolved exactly as before,
    with numpy's argpartition on their recomputed gradient rows.  The
    topology is identical to the materialised path (``fused_grow=False``).
    """

    def __init__(self, sparsity: float, drop_fraction: float = 0.3, update_freq: int = 100,
                 seed: int | None = None, capture: str = "every_step", fused_grow: bool = True):
        super().__init__(sparsity=sparsity, drop_fraction=drop_fraction, update_freq=update_freq)
        if capture not in ("every_step", "update_step"):
            raise ValueError(f"capture must be 'every_step' or 'update_step', got {capture!r}")
        self.fused_grow = bool(fused_grow)
        self._rng = np.random.default_rng(seed)
        self._captured: dict[int, dict] = {}
        self._hook_handles: list = []
        self.capture = capture
        self._generation = 0

    def _capturing(self) -> bool:
        return self.capture == "every_step" or (self._step_idx + 1) % self.update_freq == 0

    def graph_variant(self):
        """Key for a CUDA-graphed step: whether the next forward / backward
        clones X and dY, and into which generation of clone buffers (an update
        drops them, so a graph recorded before it must not be replayed after)."""
        return (self._capturing(), self._generation if self._capturing() else 0)

    def attach(self, layer) -> None:
        before = len(self.layers)
        super().attach(layer)
        if len(self.layers) == before:
            return

        def _fwd_hook(mod, inputs, output):
            if self._capturing():
                self._captured.setdefault(id(mod), {})["X"] = inputs[0].detach().clone()

        def _bwd_hook(mod, grad_input, grad_output):
            dY = grad_output[0]
            if dY is not None and self._capturing():
                self._captured.setdefault(id(mod), {})["dY"] = dY.detach().clone()

        self._hook_handles.append(layer.register_forward_hook(_fwd_hook))
        self._hook_handles.append(layer.register_full_backward_hook(_bwd_hook))

    def update(self) -> None:
        self._generation += 1
        for layer in self.layers:
            self._update_layer(layer, self._rng)

    def dense_grad(self, layer) -> torch.Tensor | None:
        """G = dY^T . X for the captured step (M x K), or None."""
        cap = self._captured.get(id(layer))
        if cap is None or "X" not in cap or "dY" not in cap:
            return None
        X_flat = cap["X"].reshape(-1, layer.in_features)
        dY_flat = cap["dY"].reshape(-1, layer.out_features)
        return dense_grad(dY_flat.t().contiguous(), X_flat.t().contiguous())

    def _operands(self, layer):
        """(dY^T [M, N], X^T [K, N]) of the captured step, or None."""
        cap = self._captured.get(id(layer))
        if cap is None or "X" not in cap or "dY" not in cap:
            return None
        X_flat = cap["X"].reshape(-1, layer.in_features)
        dY_flat = cap["dY"].reshape(-1, layer.out_features)
        return (dY_flat.t().to(torch.float32).contiguous(), X_flat.t().to(torch.float32).contiguous())

    def _update_layer(self, layer, rng, G: torch.Tensor | None = None) -> None:
        if G is None and self.fused_grow:
            ops = self._operands(layer)
            if ops is None:
                return
            if ops[0].shape[1] > 0 and layer._csr.nnz > 0:
                self._update_layer_fused(layer, *ops)
                return
        if G is None:
            G = self.dense_grad(layer)
            if G is None:
                return
        csr = layer._csr
        if csr.nnz == 0:
            self._captured.pop(id(layer), None)
            return
        _check_cols(csr)
        G = G.to(device=csr.device, dtype=torch.float32).contiguous()
        pr = _Prune(csr, self.drop_fraction)
        flags = torch.empty(csr.nrows, dtype=torch.int32, device=csr.device)
        lib = N.lib()
        s = csr._stream()
        N.call("sl_dst_apply_topk", csr._abi_ref(), N.ptr(pr.thr), N.ptr(pr.force), N.ptr(G),
                                      N.ptr(flags), s)
        flags_h = flags.cpu().numpy()
        flagged = np.nonzero((flags_h != 0) & (csr._rn_h > 0))[0]
        if flagged.size:
            self._resolve_on_host(csr, pr, G, flagged)
        pr.finish()
        self._captured.pop(id(layer), None)

    def _update_layer_fused(self, layer, dYt: torch.Tensor, Xt: torch.Tensor) -> None:
        """Prune as usual, then grow from per-tile gradient candidates (the
        M x K gradient is never stored); tie / NaN rows fall back to the
        reference's argpartition on their recomputed gradient rows."""
        csr = layer._csr
        _check_cols(csr)
        dev, s = csr.device, csr._stream()
        M, K = csr.nrows, csr.ncols
        dYt = dYt.to(dev)
        Xt = Xt.to(dev)
        Nn = dYt.shape[1]
        pr = _Prune(csr, self.drop_fraction)
        bits = torch.empty(M, (K + 31) // 32, dtype=torch.int32, device=dev)
        n_grow = torch.empty(M, dtype=torch.int32, device=dev)
        N.call("sl_rigl_prep", csr._abi_ref(), N.ptr(pr.thr), N.ptr(pr.force), N.ptr(bits),
               N.ptr(n_grow), s)
        tcols = int(N.lib().sl_rigl_tile_cols(M, K))
        lmax = int(min(int(csr._rn_h.max()) + 1, tcols))
        tiles = (K + tcols - 1) // tcols
        cand_key = torch.empty(M * tiles * lmax, dtype=torch.int32, device=dev)
        cand_col = torch.empty(M * tiles * lmax, dtype=torch.int32, device=dev)
        cand_cnt = torch.empty(M * tiles, dtype=torch.int32, device=dev)
        flags = torch.zeros(M, dtype=torch.int32, device=dev)
        N.call("sl_rigl_candidates", N.ptr(dYt), N.ptr(Xt), M, K, Nn, N.ptr(bits), N.ptr(n_grow),
               lmax, tcols, N.ptr(cand_key), N.ptr(cand_col), N.ptr(cand_cnt), N.ptr(flags), s)
        off = torch.zeros(M + 1, dtype=torch.int32, device=dev)
        total = torch.empty(1, dtype=torch.int64, device=dev)
        N.call("sl_exclusive_scan", N.ptr(n_grow), M, N.ptr(off), N.ptr(total), s)
        off[M:].copy_(total)  # grow lists of row i: [off[i], off[i + 1])
        grow = torch.empty(max(csr.nnz, 1), dtype=torch.int32, device=dev)  # >= sum(n_grow)
        mask = torch.empty(M, dtype=torch.int32, device=dev)
        N.call("sl_rigl_merge", M, K, lmax, tcols, N.ptr(cand_key), N.ptr(cand_col), N.ptr(cand_cnt),
               N.ptr(n_grow), N.ptr(off), N.ptr(csr.row_nnz), N.ptr(flags), N.ptr(mask),
               N.ptr(grow), s)
        N.call("sl_dst_apply_cols", csr._abi_ref(), N.ptr(pr.thr), N.ptr(pr.force), N.ptr(mask),
               N.ptr(off), N.ptr(grow), s)
        flags_h = flags.cpu().numpy()
        flagged = np.nonzero((flags_h != 0) & (csr._rn_h > 0))[0]
        if flagged.size:
            idx = torch.from_numpy(flagged.astype(np.int64)).to(dev)
            G_rows = dense_grad(dYt.index_select(0, idx), Xt)
            self._resolve_on_host(csr, pr, _RowsOf(G_rows, flagged), flagged)
        pr.finish()
        self._captured.pop(id(layer), None)

    @staticmethod
    def _resolve_on_host(csr, pr, G, rows) -> None:
        """Rows whose grow set is not unique: same selection as the reference
        (np.argpartition on the row's |G| with survivors at -inf)."""
        thr = np.float32(pr.thr.item())
        force = pr.force.cpu().numpy()
        mask = np.zeros(csr.nrows, np.int32)
        counts = np.zeros(csr.nrows, np.int32)
        lists = []
        for i in rows:
            i = int(i)
            s0, n = int(csr._rs_h[i]), int(csr._rn_h[i])
            lc = csr.col_indices[s0:s0 + n].cpu().numpy()
            lv = csr.values[s0:s0 + n].cpu().numpy()
            keep = np.abs(lv) > thr
            if force[i] >= 0:
                keep[force[i]] = True
            sc = lc[keep]
            n_drop = n - sc.size
            row = np.abs(G[i].cpu().numpy())
            row[sc] = -np.inf
            avail = int((row > -np.inf).sum())
            n_grow = min(n_drop, avail)
            mask[i] = 1
            if n_grow > 0:
                g = np.argpartition(-row, n_grow - 1)[:n_grow].astype(np.int32)
                lists.append(g)
                counts[i] = n_grow
        off = np.zeros(csr.nrows + 1, np.int32)
        np.cumsum(counts, out=off[1:])
        cols = np.concatenate(lists) if lists else np.zeros(1, np.int32)
        dev = csr.device
        t = [torch.from_numpy(a).to(dev) for a in (mask, off, cols)]
        N.call("sl_dst_apply_cols", csr._abi_ref(), N.ptr(pr.thr), N.ptr(pr.force),
                                          N.ptr(t[0]), N.ptr(t[1]), N.ptr(t[2]), csr._stream())


class _RowsOf:
    """G[i] for the rows computed (a subset of the layer's rows)."""

    def __init__(self, G_rows: torch.Tensor, rows):
        self.G = G_rows
        self.pos = {int(r): k for k, r in enumerate(rows)}

    def __getitem__(self, i):
        return self.G[self.pos[int(i)]]


def dense_grad(dY: torch.Tensor, X: torch.Tensor) -> torch.Tensor:
    """G[M,K] = dY[M,N] . X[K,N]^T in fp32 on the GPU
    (csrc/kernels/dense_grad.cpp:463-523, binding csrc/bindings.cpp:445-486)."""
    if dY.dim() != 2:
        raise ValueError(f"dense_grad: dY must be 2-D, got ndim={dY.dim()}.")
    if X.dim() != 2:
        raise ValueError(f"dense_grad: X must be 2-D, got ndim={X.dim()}.")
    if dY.shape[1] != X.shape[1]:
        raise ValueError(f"dense_grad: dY.shape[1]={dY.shape[1]} must equal "
                         f"X.shape[1]={X.shape[1]} (shared inner dim N).")
    dev = N.require_cuda(dY.device if dY.is_cuda else None)
    dY = dY.to(device=dev, dtype=torch.float32).contiguous()
    X = X.to(device=dev, dtype=torch.float32).contiguous()
    M, Nn = dY.shape
    K = X.shape[0]
    G = torch.empty(M, K, dtype=torch.float32, device=dev)
    N.call("sl_dense_grad", N.ptr(dY), N.ptr(X), M, K, Nn, N.ptr(G), N.stream_ptr(dev))
    return G
