"""``sparselab`` import surface over :mod:`sparsecore_b200`.

Code written against the reference package keeps its imports unchanged:
``import sparselab``, ``from sparselab.router import SET``,
``from sparselab.ops import _SpMMFunction``, ``sparselab.layout.PaddedCSR``,
``sparselab.nn.SparseLinear`` (the reference's ``sparselab/__init__.py:56-76``
exposes the same modules and names).  Every name resolves to the B200
implementation; nothing here computes.  The native ``sparselab._core``
module of the reference has no counterpart: its kernels are the C-ABI
library behind these modules.
"""
import sys as _sys

import sparsecore_b200 as _impl
from sparsecore_b200 import *  # noqa: F401,F403
from sparsecore_b200 import layout, nn, ops, router  # noqa: F401

for _name in ("layout", "nn", "ops", "router"):
    _sys.modules[__name__ + "." + _name] = getattr(_impl, _name)

__all__ = list(_impl.__all__)
__version__ = _impl.__version__
