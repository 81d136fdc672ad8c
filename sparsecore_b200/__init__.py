"""sparsecore_b200 — B200-native (sm_100a) padded-CSR sparse training.

A drop-in for the reference ``sparselab`` package's sparse-training path:

    PaddedCSR          padded-row CSR storage (CUDA memory)
    spmm(W, X)         Y = W @ X, autograd-aware (SDDMM dW, dX over W^T)
    SparseLinear       nn.Linear replacement backed by a PaddedCSR
    SparsityAlgorithm, DynamicSparsityAlgorithm, Static, SET, RigL
                       dynamic-sparsity routers (GPU prune / regrow)

``import sparsecore_b200 as sparselab`` gives the reference's names.  Every
kernel runs in the in-tree CUDA library ``_lib/libsparsecore_b200.so``
(C ABI: include/sparsecore_b200.h); there is no CPU path.
"""
import torch as _torch  # noqa: F401

from . import layout
from .layout import PaddedCSR, transpose_with_perm
from .ops import critical_path_stream, set_async_weight_grad, spmm
from .nn import SparseLinear, sparse_mlp
from .router import SparsityAlgorithm, Static, DynamicSparsityAlgorithm, SET, RigL, dense_grad
from . import torch_ops  # registers torch.ops.sparselab.spmm_fwd / sddmm_dw

__all__ = [
    "PaddedCSR",
    "spmm",
    "SparseLinear",
    "sparse_mlp",
    "SparsityAlgorithm",
    "DynamicSparsityAlgorithm",
    "Static",
    "SET",
    "RigL",
    "dense_grad",
    "transpose_with_perm",
    "critical_path_stream",
    "set_async_weight_grad",
]
__version__ = "0.1.0"
