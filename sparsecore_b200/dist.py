"""Data-parallel training over NCCL for models with SparseLinear layers.

The reference has no distributed path; this adds the one the benchmark
needs.  Every rank holds a full replica with the same topology; the batch is
sharded.  Per step:

* ``allreduce_grads()`` -- the live-slot gradients of every SparseLinear
  (packed out of the padded ``total_capacity`` layout by ``sl_pack_live``;
  padding never travels) and all dense gradients are concatenated into one
  flat fp32 buffer, all-reduced with ReduceOp.AVG and scattered back
  (``sl_unpack_live``).  With ``overlap=True`` (and the library's async
  weight-gradient mode on) the sparse part is split into buckets of about
  ``bucket_mb`` in backward order; each layer's gradient is packed on the
  weight-gradient side stream as soon as its SDDMM is enqueued, and a
  bucket's all-reduce is launched there when its last layer is packed, so
  the exchange runs while the rest of the backward pass does.
  ``allreduce_grads()`` then only waits for the buckets, unpacks them and
  exchanges the small dense part.
* after a router update, ``broadcast_topology(src=0)`` sends rank 0's
  ``col_indices`` / ``row_nnz`` / ``values`` of every layer (one flat int32
  and one flat fp32 broadcast) plus the topology versions, so all replicas
  hold the same mask even when the grow decision uses rank-local data
  (RigL's dense gradient).
* ``topology_checksum()`` all-gathers a per-rank checksum of the masks to
  detect divergence.

Host-side planning (bucket offsets, which tensors travel) is independent of
the device kernels; ``pack`` / ``unpack`` can be swapped (tests on CPU gloo
ranks use index-based stand-ins).
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Callable

import torch
import torch.distributed as dist

from . import _native as N
from . import ops


@dataclass
class _Slot:
    kind: str          # "sparse" | "dense"
    module: object     # SparseLinear for sparse
    param: torch.Tensor
    offset: int
    length: int


def _gpu_pack(layer, offsets: torch.Tensor, src: torch.Tensor, dst: torch.Tensor) -> None:
    csr = layer._csr
    N.call("sl_pack_live", csr._abi_ref(), N.ptr(offsets), N.ptr(src), N.ptr(dst),
                                 csr._stream())


def _gpu_unpack(layer, offsets: torch.Tensor, src: torch.Tensor, dst: torch.Tensor) -> None:
    csr = layer._csr
    N.call("sl_unpack_live", csr._abi_ref(), N.ptr(offsets), N.ptr(src), N.ptr(dst), 1.0,
                                   csr._stream())


def _gpu_offsets(layer) -> torch.Tensor:
    csr = layer._csr
    out = torch.empty(csr.nrows, dtype=torch.int32, device=csr.device)
    total = torch.empty(1, dtype=torch.int64, device=csr.device)
    N.call("sl_exclusive_scan", N.ptr(csr.row_nnz), csr.nrows, N.ptr(out), N.ptr(total),
                                      csr._stream())
    return out


class SparseDataParallel:
    """Gradient / topology synchronisation for a replicated model."""

    def __init__(self, model: torch.nn.Module, process_group=None,
                 pack: Callable | None = None, unpack: Callable | None = None,
                 offsets: Callable | None = None, sparse_layers: list | None = None,
                 overlap: bool = False, bucket_mb: float = 8.0):
        from .nn import SparseLinear

        self.model = model
        self.pg = process_group
        self.sparse_layers = (list(sparse_layers) if sparse_layers is not None else
                              [m for m in model.modules() if isinstance(m, SparseLinear)])
        sparse_ids = {id(m._values) for m in self.sparse_layers}
        self.dense_params = [p for p in model.parameters()
                             if p.requires_grad and id(p) not in sparse_ids]
        self._pack = pack or _gpu_pack
        self._unpack = unpack or _gpu_unpack
        self._offsets_fn = offsets or _gpu_offsets
        self._plan_key = None
        self._plan: list[_Slot] = []
        self._bucket: torch.Tensor | None = None
        self._offsets: dict[int, torch.Tensor] = {}
        # overlapped exchange state
        self.overlap = bool(overlap)
        self.bucket_bytes = int(bucket_mb * 2 ** 20)
        self._slot_of: dict[int, _Slot] = {}      # id(param) -> slot
        self._bucket_of: dict[int, int] = {}      # id(param) -> bucket index
        self._bucket_ranges: list[tuple[int, int, int]] = []  # (offset, length, n_layers)
        self._packed: dict[int, int] = {}         # bucket -> layers packed this step
        self._works: list = []
        self._packed_params: set = set()
        if self.overlap:
            from . import ops

            ops.add_weight_grad_hook(self._on_weight_grad)

    # ── planning ────────────────────────────────────────────────────────
    def _key(self):
        return tuple((m._csr.topology_version, m._csr.nnz) for m in self.sparse_layers)

    def plan(self) -> list[_Slot]:
        key = self._key()
        if key == self._plan_key:
            return self._plan
        slots, off = [], 0
        # Sparse layers in backward order (their gradients arrive in that
        # order), then the dense parameters; buckets are contiguous ranges.
        self._bucket_ranges, self._bucket_of, self._slot_of = [], {}, {}
        b_off, b_len, b_n = 0, 0, 0
        for m in reversed(self.sparse_layers):
            sl = _Slot("sparse", m, m._values, off, m._csr.nnz)
            slots.append(sl)
            self._slot_of[id(m._values)] = sl
            self._bucket_of[id(m._values)] = len(self._bucket_ranges)
            off += m._csr.nnz
            b_len += m._csr.nnz
            b_n += 1
            if 4 * b_len >= self.bucket_bytes:
                self._bucket_ranges.append((b_off, b_len, b_n))
                b_off, b_len, b_n = off, 0, 0
        if b_n:
            self._bucket_ranges.append((b_off, b_len, b_n))
        for p in self.dense_params:
            slots.append(_Slot("dense", None, p, off, p.numel()))
            off += p.numel()
        dev = slots[0].param.device if slots else torch.device("cpu")
        if self._bucket is None or self._bucket.numel() != off:
            self._bucket = torch.empty(off, dtype=torch.float32, device=dev)
        self._offsets = {id(m): self._offsets_fn(m) for m in self.sparse_layers}
        self._plan, self._plan_key = slots, key
        return slots

    @property
    def bucket_numel(self) -> int:
        return sum(s.length for s in self.plan())

    # ── per-step gradient exchange ──────────────────────────────────────
    def world_size(self) -> int:
        return dist.get_world_size(self.pg) if dist.is_available() and dist.is_initialized() else 1

    # ── overlapped exchange ─────────────────────────────────────────────
    def _on_weight_grad(self, param, dW) -> None:
        """Called on the weight-gradient side stream right after a layer's
        SDDMM: pack its live slots into its bucket and, once the bucket is
        complete, launch the bucket's all-reduce there."""
        if self.world_size() == 1 or torch.cuda.is_current_stream_capturing():
            return
        self.plan()
        sl = self._slot_of.get(id(param))
        if sl is None:
            return
        b = self._bucket_of[id(param)]
        off, length, n = self._bucket_ranges[b]
        self._pack(sl.module, self._offsets[id(sl.module)], dW, self._bucket[sl.offset:sl.offset + sl.length])
        self._packed_params.add(id(param))
        self._packed[b] = self._packed.get(b, 0) + 1
        if self._packed[b] == n:
            view = self._bucket[off:off + length]
            if dist.get_backend(self.pg) == "nccl":
                w = dist.all_reduce(view, op=dist.ReduceOp.AVG, group=self.pg, async_op=True)
            else:
                w = dist.all_reduce(view, op=dist.ReduceOp.SUM, group=self.pg, async_op=True)
            self._works.append((w, view))

    def _finish_overlapped(self, slots, world) -> bool:
        """Wait for the buckets launched during backward and unpack them; the
        dense part goes through one all-reduce here.  False when the
        backward did not pack every sparse layer (e.g. the synchronous
        weight-gradient mode): the caller then exchanges everything."""
        sparse = [s for s in slots if s.kind == "sparse"]
        ok = len(self._packed_params) == len(sparse) and len(self._works) == len(self._bucket_ranges)
        if not ok:
            for w, _ in self._works:
                w.wait()
            self._works, self._packed, self._packed_params = [], {}, set()
            return False
        nccl = dist.get_backend(self.pg) == "nccl"
        for w, view in self._works:
            w.wait()
            if not nccl:
                view.div_(world)
        for s in sparse:
            view = self._bucket[s.offset:s.offset + s.length]
            if s.param.grad is None:
                s.param.grad = torch.zeros_like(s.param)
            self._unpack(s.module, self._offsets[id(s.module)], view, s.param.grad)
        self._works, self._packed, self._packed_params = [], {}, set()
        dense = [s for s in slots if s.kind == "dense"]
        if dense:
            d0 = dense[0].offset
            buf = self._bucket[d0:]
            for s in dense:
                view = self._bucket[s.offset:s.offset + s.length]
                view.copy_(s.param.grad.reshape(-1)) if s.param.grad is not None else view.zero_()
            if nccl:
                dist.all_reduce(buf, op=dist.ReduceOp.AVG, group=self.pg)
            else:
                dist.all_reduce(buf, op=dist.ReduceOp.SUM, group=self.pg)
                buf.div_(world)
            for s in dense:
                view = self._bucket[s.offset:s.offset + s.length]
                if s.param.grad is None:
                    s.param.grad = torch.zeros_like(s.param)
                s.param.grad.copy_(view.view_as(s.param.grad))
        return True

    def allreduce_grads(self) -> None:
        world = self.world_size()
        if world == 1:
            return
        slots = self.plan()
        if self.overlap and (self._works or self._packed_params):
            if self._finish_overlapped(slots, world):
                return
        if self._pack is _gpu_pack and self._unpack is _gpu_unpack:
            self._exchange_batched(slots, world)
            return
        buf = self._bucket
        for s in slots:
            view = buf[s.offset:s.offset + s.length]
            g = s.param.grad
            if s.kind == "sparse":
                if g is None:
                    view.zero_()
                else:
                    self._pack(s.module, self._offsets[id(s.module)], g, view)
            else:
                view.copy_(g.reshape(-1)) if g is not None else view.zero_()
        if dist.get_backend(self.pg) == "nccl":
            dist.all_reduce(buf, op=dist.ReduceOp.AVG, group=self.pg)
        else:
            dist.all_reduce(buf, op=dist.ReduceOp.SUM, group=self.pg)
            buf.div_(world)
        for s in slots:
            view = buf[s.offset:s.offset + s.length]
            if s.param.grad is None:
                s.param.grad = torch.zeros_like(s.param)
            if s.kind == "sparse":
                self._unpack(s.module, self._offsets[id(s.module)], view, s.param.grad)
            else:
                s.param.grad.copy_(view.view_as(s.param.grad))

    def _live_descs(self, sparse) -> tuple[torch.Tensor, int]:
        """Device table of sl_live_desc for the sparse slots (their current
        .grad tensors) and the launch's block count."""
        import numpy as np

        rows, blocks = [], 0
        for s in sparse:
            csr = s.module._csr
            rows.append((csr.row_start.data_ptr(), csr.row_nnz.data_ptr(),
                         self._offsets[id(s.module)].data_ptr(), s.param.grad.data_ptr(),
                         csr.nrows, s.offset, blocks))
            blocks += (csr.nrows + 7) // 8
        arr = np.array(rows, dtype=np.int64).reshape(-1)
        return torch.from_numpy(arr).to(self._bucket.device), blocks

    def _exchange_batched(self, slots, world) -> None:
        """The exchange with one pack launch for every sparse layer, one
        concatenation of the dense gradients, one all-reduce, one unpack
        launch and one multi-tensor copy back (instead of a pack, a copy and
        an unpack per tensor)."""
        buf = self._bucket
        sparse = [s for s in slots if s.kind == "sparse"]
        dense = [s for s in slots if s.kind == "dense"]
        for s in sparse:
            if s.param.grad is None:
                s.param.grad = torch.zeros_like(s.param)
        stream = N.stream_ptr(buf.device)
        descs, blocks = self._live_descs(sparse) if sparse else (None, 0)
        if sparse:
            N.call("sl_pack_live_batch", N.ptr(descs), len(sparse), blocks, N.ptr(buf), stream)
        if dense:
            d0 = dense[0].offset
            torch.cat([s.param.grad.reshape(-1) if s.param.grad is not None
                       else torch.zeros(s.length, device=buf.device) for s in dense],
                      out=buf[d0:d0 + sum(s.length for s in dense)])
        if dist.get_backend(self.pg) == "nccl":
            dist.all_reduce(buf, op=dist.ReduceOp.AVG, group=self.pg)
        else:
            dist.all_reduce(buf, op=dist.ReduceOp.SUM, group=self.pg)
            buf.div_(world)
        if sparse:
            N.call("sl_unpack_live_batch", N.ptr(descs), len(sparse), blocks, N.ptr(buf), stream)
        if dense:
            for s in dense:
                if s.param.grad is None:
                    s.param.grad = torch.zeros_like(s.param)
            torch._foreach_copy_([s.param.grad.view(-1) for s in dense],
                                 [buf[s.offset:s.offset + s.length] for s in dense])

    # ── topology synchronisation ────────────────────────────────────────
    def broadcast_topology(self, src: int = 0) -> None:
        """Make every replica's masks (and values) equal to rank ``src``'s."""
        if self.world_size() == 1 or not self.sparse_layers:
            return
        ints = torch.cat([torch.cat([m._csr.col_indices, m._csr.row_nnz]) for m in self.sparse_layers])
        flts = torch.cat([m._csr.values for m in self.sparse_layers])
        vers = torch.tensor([m._csr.topology_version for m in self.sparse_layers],
                            dtype=torch.int64, device=ints.device)
        for t in (ints, flts, vers):
            dist.broadcast(t, src=src, group=self.pg)
        io = fo = 0
        for m, v in zip(self.sparse_layers, vers.tolist()):
            csr = m._csr
            cap, M = csr.total_capacity, csr.nrows
            with torch.no_grad():
                csr.col_indices.copy_(ints[io:io + cap])
                csr.row_nnz.copy_(ints[io + cap:io + cap + M])
                csr.values.copy_(flts[fo:fo + cap])
            io += cap + M
            fo += cap
            csr._sync_row_nnz_from_device()
            csr.topology_version_ = int(v)
            # The cached W^T is keyed by topology_version only; a rank whose
            # own mask differed at the same version would otherwise keep
            # using a W^T (and perm) of its old mask for dX.
            ops._transpose_cache.pop(id(csr), None)

    def topology_checksum(self) -> list[int]:
        """All ranks' mask checksums (equal when the replicas agree)."""
        h = 0
        for m in self.sparse_layers:
            c = m._csr.col_indices.to(torch.int64)
            idx = torch.arange(c.numel(), device=c.device, dtype=torch.int64)
            h = (h * 1000003 + int(((c + 7) * (idx % 65521 + 1)).sum().item())) % (2 ** 61 - 1)
        t = torch.tensor([h], dtype=torch.int64,
                         device=self.sparse_layers[0]._csr.device if self.sparse_layers else "cpu")
        if self.world_size() == 1:
            return [int(t.item())]
        out = [torch.zeros_like(t) for _ in range(self.world_size())]
        dist.all_gather(out, t, group=self.pg)
        return [int(x.item()) for x in out]


def sync_after_router_step(ddp: SparseDataParallel, algo, src: int = 0) -> bool:
    """Broadcast the topology if ``algo.step()`` just ran an update."""
    if getattr(algo, "last_update_step", None) == getattr(algo, "_step_idx", -1):
        ddp.broadcast_topology(src)
        return True
    return False


