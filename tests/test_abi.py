"""The C-ABI library loads and exports every symbol the header declares.
CPU only: no compute call is made."""
import os
import re

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(REPO, "include", "sparsecore_b200.h")


def declared_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"^SL_API\s+[\w\s\*]+?\b(sl_\w+)\s*\(", text, flags=re.M)))


def test_header_declares_entry_points():
    syms = declared_symbols()
    assert "sl_spmm_fwd" in syms and "sl_sddmm_dw" in syms and "sl_transpose_fill" in syms
    assert len(syms) >= 20


def test_library_exports_every_declared_symbol():
    from sparsecore_b200 import _native as N
    from sparsecore_b200.build import build

    build()
    lib = N.load_library()
    for s in declared_symbols():
        assert hasattr(lib, s), s
        assert s in N.SIGNATURES, f"{s} has no ctypes signature"


def test_library_metadata_calls_without_gpu():
    from sparsecore_b200 import _native as N

    lib = N.load_library()
    assert lib.sl_version().startswith(b"sparsecore_b200")
    assert lib.sl_dst_max_ncols() >= 16384
    assert lib.sl_transpose_scratch_bytes(4096, 4096) == 128 * 4096 * 4
    assert lib.sl_dst_scratch_bytes() >= 1024


def test_product_fails_loudly_without_cuda():
    import torch

    if torch.cuda.is_available():
        pytest.skip("has a GPU")
    import sparsecore_b200 as sl

    with pytest.raises(RuntimeError, match="CUDA"):
        sl.SparseLinear(8, 4)
    with pytest.raises(RuntimeError, match="CUDA"):
        sl.PaddedCSR(2, 2)


def test_product_never_imports_oracle():
    pkg = os.path.join(REPO, "sparsecore_b200")
    for root, _, files in os.walk(pkg):
        for f in files:
            if f.endswith(".py"):
                src = open(os.path.join(root, f)).read()
                assert "oracle" not in src.replace("oracle-free", ""), f


def test_sparselab_import_surface():
    """The reference's import paths resolve to this implementation."""
    import sparselab
    import sparselab.layout
    import sparselab.nn
    import sparselab.ops
    import sparselab.router
    from sparselab.ops import _SpMMFunction, _cached_transpose, _clear_transpose_cache, spmm  # noqa: F401
    from sparselab.router import SET, RigL, Static  # noqa: F401

    import sparsecore_b200

    assert sparselab.PaddedCSR is sparsecore_b200.PaddedCSR
    assert sparselab.SparseLinear is sparsecore_b200.SparseLinear
    assert sparselab.spmm is sparsecore_b200.spmm
    assert sparselab.router.RigL is sparsecore_b200.RigL
    assert sparselab.layout.transpose_with_perm is sparsecore_b200.transpose_with_perm
