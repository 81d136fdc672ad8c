"""CUDA-graph replay of a whole training step.

A sparse training step launches a few hundred small kernels (SpMM, SDDMM,
transposes, the cached-transpose refresh, the optimizer); for small models
the host cost of those launches exceeds the GPU work.  ``GraphedStep``
captures one step -- forward, backward, gradient exchange and optimizer, as
written in the caller's ``step_fn`` -- into a CUDA graph over static input
buffers and replays it.

Topology changes (a SET / RigL update, a checkpoint load) rebuild each
layer's cached transpose, whose buffers the graph would otherwise keep
using, so the step is re-captured whenever any SparseLinear's
``topology_version`` differs from the captured one; the transposes are
rebuilt eagerly first (capture records, it does not execute).

Requirements on ``step_fn``: it starts with ``optimizer.zero_grad(
set_to_none=True)``, reads its inputs only from the static tensors given
here, returns the loss tensor, and contains no host synchronisation (no
``.item()``); the optimizer must be capturable (``AdamW(...,
capturable=True)``; plain SGD is).  The step must have run eagerly at least
once before the first capture (lazy library initialisation).  Router steps
stay outside the graph.

``variant`` (optional) is a callable returning a hashable key for steps
whose recorded work differs: RigL with ``capture="update_step"`` clones its
inputs only before an update, so ``variant=algo.graph_variant`` keeps two
graphs, one with the clones and one without, and replays the one the next
step needs.  All variants are dropped on a topology change.
"""
from __future__ import annotations

import torch

from . import _native as N
from . import ops
from .nn import SparseLinear

__all__ = ["GraphedStep"]


class GraphedStep:
    def __init__(self, model: torch.nn.Module, step_fn, static_inputs: tuple, variant=None):
        self.model = model
        self.step_fn = step_fn
        self.inputs = tuple(static_inputs)
        self.variant = variant
        self.layers = [m for m in model.modules() if isinstance(m, SparseLinear)]
        self._graphs: dict = {}  # variant key -> (graph, loss, launches)
        self._key = None
        self.graph: torch.cuda.CUDAGraph | None = None
        self.loss: torch.Tensor | None = None
        self.captures = 0
        self.launches_per_replay = 0  # this library's kernels inside the last graph replayed

    def _topology(self):
        return tuple((id(m._csr), m._csr.topology_version) for m in self.layers)

    def _variant(self):
        return self.variant() if self.variant is not None else None

    def capture(self) -> None:
        """Capture the step for the current variant (re-capturing all of them
        from scratch if the topology changed)."""
        if self._topology() != self._key:
            self._graphs.clear()  # release the previous graphs' memory first
            self.graph = None
        for m in self.layers:
            ops._cached_transpose(m._csr)  # rebuild (eagerly) before recording
        self.check_status()
        v = self._variant()
        self._graphs.pop(v, None)
        g = torch.cuda.CUDAGraph()
        l0 = N.launches["count"]
        with torch.cuda.graph(g):
            loss = self.step_fn(*self.inputs)
        launches = N.launches["count"] - l0
        N.launches["count"] = l0
        self._graphs[v] = (g, loss, launches)
        self._key = self._topology()
        self.captures += 1

    def check_status(self) -> None:
        """Synchronise and raise RuntimeError if a bounded device-side wait
        gave up since the last check (the replays since then produced
        incomplete gradients).  Runs at every (re-)capture; call it at any
        other point that synchronises, e.g. where the loss is read."""
        devs = {m._csr.values.device for m in self.layers} or {torch.device("cuda", torch.cuda.current_device())}
        for dev in devs:
            N.check_device_status(dev)

    def __call__(self) -> torch.Tensor:
        v = self._variant()
        if self._topology() != self._key or v not in self._graphs:
            self.capture()
        self.graph, self.loss, self.launches_per_replay = self._graphs[v]
        self.graph.replay()
        N.launches["count"] += self.launches_per_replay
        return self.loss
