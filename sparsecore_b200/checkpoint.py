"""Checkpoints that carry the sparse topology and the router state.

The reference serialises only ``SparseLinear._values`` and the bias; the mask
(``col_indices`` / ``row_nnz``) is not saved, so a resumed run must rebuild
the layer from the same seed and cannot resume after a SET / RigL update
(``tests/test_sparse_linear.py:312-333`` of the reference).  ``save`` /
``load`` here add, per SparseLinear, the padded-CSR structure arrays and
``topology_version``, and for a router its step counter and its numpy
``Generator`` state.  A run resumed from one of these checkpoints continues
exactly where it stopped: same masks, same values, same optimizer moments,
same future random draws.

Format (one ``torch.save`` dict):
    {"format": "sparsecore_b200.checkpoint/1",
     "model": model.state_dict(),
     "topology": {module_name: {"shape", "row_start", "row_nnz", "row_capacity",
                                "col_indices", "topology_version"}},
     "optimizer": optimizer.state_dict() | None,
     "router": {"type", "step_idx", "last_update_step", "rng"} | None,
     "extra": anything the caller passes}
"""
from __future__ import annotations

import torch

from .nn import SparseLinear

__all__ = ["save", "load", "topology_state", "router_state", "load_router_state"]

FORMAT = "sparsecore_b200.checkpoint/1"


def topology_state(model: torch.nn.Module) -> dict:
    """Structure arrays of every SparseLinear in ``model`` (CPU tensors)."""
    out = {}
    for name, m in model.named_modules():
        if isinstance(m, SparseLinear):
            c = m._csr
            out[name] = {
                "shape": (c.nrows, c.ncols),
                "row_start": c.row_start.detach().cpu().clone(),
                "row_nnz": c.row_nnz.detach().cpu().clone(),
                "row_capacity": c.row_capacity.detach().cpu().clone(),
                "col_indices": c.col_indices.detach().cpu().clone(),
                "topology_version": int(c.topology_version),
            }
    return out


def router_state(algorithm) -> dict | None:
    """Step counter and random-generator state of a sparsity algorithm."""
    if algorithm is None:
        return None
    rng = getattr(algorithm, "_rng", None)
    return {
        "type": type(algorithm).__name__,
        "step_idx": int(algorithm._step_idx),
        "last_update_step": getattr(algorithm, "last_update_step", None),
        "rng": rng.bit_generator.state if rng is not None else None,
    }


def load_router_state(algorithm, state: dict | None) -> None:
    if algorithm is None or state is None:
        return
    if state["type"] != type(algorithm).__name__:
        raise ValueError(f"checkpoint router is {state['type']}, got {type(algorithm).__name__}")
    algorithm._step_idx = int(state["step_idx"])
    if hasattr(algorithm, "last_update_step"):
        algorithm.last_update_step = state["last_update_step"]
    if state["rng"] is not None:
        algorithm._rng.bit_generator.state = state["rng"]


def save(path, model: torch.nn.Module, optimizer=None, algorithm=None, extra=None) -> None:
    torch.save({
        "format": FORMAT,
        "model": model.state_dict(),
        "topology": topology_state(model),
        "optimizer": optimizer.state_dict() if optimizer is not None else None,
        "router": router_state(algorithm),
        "extra": extra,
    }, path)


def _restore_topology(layer: SparseLinear, t: dict) -> None:
    from . import ops
    from .layout import PaddedCSR

    c = layer._csr
    if tuple(t["shape"]) != (c.nrows, c.ncols):
        raise ValueError(f"checkpoint layer shape {tuple(t['shape'])} != model's {(c.nrows, c.ncols)}")
    dev = c.device
    same_layout = (torch.equal(t["row_start"], c.row_start.cpu())
                   and torch.equal(t["row_capacity"], c.row_capacity.cpu()))
    with torch.no_grad():
        if same_layout:
            # In place: the Parameter keeps aliasing the CSR value storage.
            c.col_indices.copy_(t["col_indices"].to(dev))
            c.row_nnz.copy_(t["row_nnz"].to(dev))
            c._sync_row_nnz_from_device()
        else:
            # Different per-row capacities: rebuild the CSR and re-point the
            # Parameter's data at the new value storage (same Parameter object,
            # so the optimizer's param references stay valid).
            cap = int(t["col_indices"].numel())
            new = PaddedCSR(c.nrows, c.ncols, torch.zeros(cap), t["col_indices"], t["row_start"],
                            t["row_nnz"], t["row_capacity"], device=dev)
            layer._csr = new
            layer._values.data = new.values
            c = new
    c.topology_version_ = int(t["topology_version"])
    ops._transpose_cache.pop(id(c), None)


def load(path, model: torch.nn.Module, optimizer=None, algorithm=None):
    """Restore a checkpoint written by ``save`` into ``model`` (and the
    optimizer / router if given).  Returns the ``extra`` payload."""
    ck = torch.load(path, map_location="cpu", weights_only=False)
    if ck.get("format") != FORMAT:
        raise ValueError(f"not a {FORMAT} checkpoint")
    layers = {name: m for name, m in model.named_modules() if isinstance(m, SparseLinear)}
    if set(layers) != set(ck["topology"]):
        raise ValueError("checkpoint SparseLinear layers do not match the model's: "
                         f"{sorted(set(layers) ^ set(ck['topology']))}")
    for name, layer in layers.items():
        _restore_topology(layer, ck["topology"][name])
    model.load_state_dict(ck["model"])
    if optimizer is not None and ck["optimizer"] is not None:
        optimizer.load_state_dict(ck["optimizer"])
    load_router_state(algorithm, ck["router"])
    return ck["extra"]
