"""The batched live-slot pack / unpack (one launch for many layers) against
the per-layer entry points, on one GPU: same packed bucket, and unpacking
restores every live slot while leaving padding untouched."""
import numpy as np
import pytest
import torch

from gpu_helpers import dev

pytestmark = pytest.mark.gpu


def test_pack_unpack_batch_matches_per_layer():
    import sparsecore_b200 as sl
    from sparsecore_b200 import _native as N
    from sparsecore_b200.dist import _gpu_offsets, _gpu_pack

    torch.manual_seed(2)
    layers = [sl.SparseLinear(70, 300, sparsity=0.8, device=dev()),
              sl.SparseLinear(300, 9, sparsity=0.5, device=dev()),
              sl.SparseLinear(1000, 17, sparsity=0.95, device=dev())]
    grads = [torch.randn(m._csr.total_capacity, device=dev()) for m in layers]
    offs = [_gpu_offsets(m) for m in layers]
    total = sum(m._csr.nnz for m in layers)
    ref = torch.empty(total + 5, device=dev())
    o = 5
    rows, blocks = [], 0
    for m, g, off in zip(layers, grads, offs):
        _gpu_pack(m, off, g, ref[o:o + m._csr.nnz])
        csr = m._csr
        rows.append((csr.row_start.data_ptr(), csr.row_nnz.data_ptr(), off.data_ptr(), g.data_ptr(),
                     csr.nrows, o, blocks))
        blocks += (csr.nrows + 7) // 8
        o += csr.nnz
    descs = torch.from_numpy(np.array(rows, dtype=np.int64).reshape(-1)).to(dev())
    s = N.stream_ptr(dev())
    got = torch.full_like(ref, 7.0)
    N.call("sl_pack_live_batch", N.ptr(descs), len(layers), blocks, N.ptr(got), s)
    assert torch.equal(got[5:], ref[5:]) and bool((got[:5] == 7.0).all())
    # unpack a scaled bucket back: live slots take the bucket's values, padding stays
    before = [g.clone() for g in grads]
    got.mul_(3.0)
    N.call("sl_unpack_live_batch", N.ptr(descs), len(layers), blocks, N.ptr(got), s)
    for m, g, b in zip(layers, grads, before):
        live = m._csr.col_indices >= 0
        assert torch.equal(g[live], b[live] * 3.0)
        assert torch.equal(g[~live], b[~live])
