"""``SparseLinear``: drop-in ``nn.Linear`` with a padded-CSR weight on a CUDA
device (mirrors sparselab/nn.py:36-268).

Initialisation reproduces the reference draw for draw (nn.py:113-185): the
sparsity-compensated Kaiming-uniform dense matrix and the ``rand >= sparsity``
mask come from torch's global CPU generator, so ``torch.manual_seed(s)``
gives the same weights and bias as the reference; the result is then built
into a PaddedCSR on the device.  ``_values`` is an ``nn.Parameter`` that
*aliases* ``_csr.values`` (same CUDA storage): optimizer updates are seen by
the kernels and router rewrites are seen by the optimizer.
"""
from __future__ import annotations

import math

import torch
import torch.nn as nn

from . import _native as N
from .layout import PaddedCSR, from_dense
from .ops import _SparseLinearFunction, _SparseMLPFunction

__all__ = ["SparseLinear", "sparse_mlp"]


class SparseLinear(nn.Module):
    """``y = x @ W^T + b`` with W (out_features x in_features) stored as a
    PaddedCSR at the requested sparsity.

    Args follow the reference: ``in_features, out_features, bias=True,
    sparsity=0.9, padding_ratio=0.2``; ``device`` (default: current CUDA
    device) picks the GPU.
    """

    def __init__(self, in_features: int, out_features: int, bias: bool = True,
                 sparsity: float = 0.9, padding_ratio: float = 0.2, device=None):
        super().__init__()
        if not (0.0 <= sparsity < 1.0):
            raise ValueError(f"sparsity must be in [0.0, 1.0), got {sparsity}")
        self.in_features = in_features
        self.out_features = out_features
        self.sparsity = sparsity
        self.padding_ratio = padding_ratio
        self._device = N.require_cuda(device)
        self._csr, values_param = self._build_csr_and_parameter(sparsity)
        self._values = values_param
        if bias:
            self.bias = nn.Parameter(torch.empty(out_features))
        else:
            self.register_parameter("bias", None)
        if self.bias is not None:
            effective_fan_in = max(1.0, in_features * (1.0 - sparsity))
            bound = 1.0 / math.sqrt(effective_fan_in)
            nn.init.uniform_(self.bias, -bound, bound)
            self.bias.data = self.bias.data.to(self._device)

    def _build_csr_and_parameter(self, sparsity: float) -> tuple[PaddedCSR, nn.Parameter]:
        effective_fan_in = max(1.0, self.in_features * (1.0 - sparsity))
        bound = 1.0 / math.sqrt(effective_fan_in)
        W_dense = torch.empty(self.out_features, self.in_features)
        nn.init.uniform_(W_dense, -bound, bound)
        mask = torch.rand(self.out_features, self.in_features) >= sparsity
        W_dense = W_dense * mask.float()
        csr = from_dense(W_dense, padding_ratio=self.padding_ratio, device=self._device)
        return csr, nn.Parameter(csr.values)

    def reset_parameters(self) -> None:
        """Redraw mask, values and bias (nn.py:187-205).  The Parameter object
        is kept; its data is rebound to the new CSR's value storage."""
        self._csr, new_values = self._build_csr_and_parameter(self.sparsity)
        with torch.no_grad():
            self._values.data = new_values.data
        if self.bias is not None:
            bound = 1.0 / math.sqrt(self.in_features)
            b = torch.empty(self.out_features)
            nn.init.uniform_(b, -bound, bound)
            with torch.no_grad():
                self.bias.copy_(b.to(self.bias.device))

    def _apply(self, fn, recurse=True):
        # Moving / casting the module must not break the values aliasing.
        before = self._values.data
        out = super()._apply(fn, recurse)
        if self._values.data.data_ptr() != before.data_ptr():
            raise RuntimeError(
                "SparseLinear: its weight lives in a device PaddedCSR and cannot be moved or "
                "cast with .to()/.cuda()/.double(); build the layer on the target device.")
        return out

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        orig_shape = x.shape
        if orig_shape[-1] != self.in_features:
            raise ValueError(f"SparseLinear expects input last dim {self.in_features}, "
                             f"got {orig_shape[-1]}")
        x_flat = x.reshape(-1, self.in_features)
        # The bias add is fused into the output transpose (nn.py:239-241).
        y_flat = _SparseLinearFunction.apply(self._values, self._csr, x_flat, self.bias)
        return y_flat.reshape(orig_shape[:-1] + (self.out_features,))

    @property
    def nnz(self) -> int:
        return self._csr.nnz

    @property
    def density(self) -> float:
        return self.nnz / (self.out_features * self.in_features)

    def extra_repr(self) -> str:
        return (f"in_features={self.in_features}, out_features={self.out_features}, "
                f"bias={self.bias is not None}, sparsity={self.sparsity}, nnz={self.nnz}")


def _plain(layer: SparseLinear) -> bool:
    return (not layer._forward_hooks and not layer._forward_pre_hooks
            and not layer._backward_hooks and not getattr(layer, "_backward_pre_hooks", None)
            and (layer.bias is None or (layer.bias.dtype == torch.float32
                                        and layer.bias.device == layer._csr.device)))


def sparse_mlp(x: torch.Tensor, fc1: SparseLinear, fc2: SparseLinear,
               activation: str = "gelu") -> torch.Tensor:
    """``fc2(act(fc1(x)))`` for two SparseLinears with ``activation`` in
    {"gelu", "relu"}.  When neither layer carries module hooks (RigL's
    gradient capture uses hooks), the hidden activation stays in the
    kernels' column-per-token layout (``ops._SparseMLPFunction``), with
    fc1's bias and the activation fused into its forward kernel and fc2's
    bias into the output transpose; otherwise the two layers are called as
    modules.  Same values either way.
    """
    if activation not in ("gelu", "relu"):
        raise ValueError(f"sparse_mlp: activation must be 'gelu' or 'relu', got {activation!r}")
    if fc1.out_features != fc2.in_features:
        raise ValueError(f"sparse_mlp: fc1.out_features={fc1.out_features} != "
                         f"fc2.in_features={fc2.in_features}")
    if not (_plain(fc1) and _plain(fc2)) or x.shape[-1] != fc1.in_features:
        h = fc1(x)
        h = torch.nn.functional.gelu(h) if activation == "gelu" else torch.relu(h)
        return fc2(h)
    shp = x.shape
    y = _SparseMLPFunction.apply(fc1._values, fc2._values, x.reshape(-1, fc1.in_features),
                                 fc1._csr, fc2._csr, activation, fc1.bias, fc2.bias)
    return y.reshape(shp[:-1] + (fc2.out_features,))
