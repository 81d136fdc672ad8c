"""sl_transpose_with_perm_noalloc: the transpose entry point that allocates
nothing, for callers that cannot call cudaMalloc (code inside a memory pool
or allocator hook, loops that forbid allocation, hosts that own all device
memory).  Its scratch is a fixed 4 MiB device array inside the library.

Checked through the C ABI against the allocating pair
sl_transpose_count / sl_transpose_fill (bit-exact: the transpose is integer
index work plus value copies), on two calls in a row with different
matrices, so the second call runs on the scratch the first one left behind.

The file name sorts last so that a stop-at-first-failure run has already run
every other test before this one.
"""
import ctypes
import math

import pytest
import torch

pytestmark = pytest.mark.gpu


def _reference_transpose(W, opp):
    import sparsecore_b200 as sl

    WT, perm = sl.transpose_with_perm(W, padding_ratio=opp - 1.0)
    return WT, perm


def _noalloc_transpose(W, opp):
    from sparsecore_b200 import _native as N

    dev = W.device
    M, K = W.nrows, W.ncols
    bound = int(math.floor(opp * W.total_capacity)) + K + 2
    rows = torch.empty(3, K, dtype=torch.int32, device=dev)
    vals = torch.full((bound,), 7.0, dtype=torch.float32, device=dev)
    cols = torch.full((bound,), 7, dtype=torch.int32, device=dev)
    perm = torch.full((bound,), 7, dtype=torch.int64, device=dev)
    total = torch.zeros(1, dtype=torch.int64, device=dev)
    WT = N.SlCsr(K, M, bound, vals.data_ptr(), cols.data_ptr(), rows[2].data_ptr(),
                 rows[0].data_ptr(), rows[1].data_ptr())
    rc = N.lib().sl_transpose_with_perm_noalloc(W._abi_ref(), opp, ctypes.byref(WT),
                                                N.ptr(perm), N.ptr(total), W._stream())
    N.check(rc, "sl_transpose_with_perm_noalloc")
    torch.cuda.synchronize()
    return rows, vals, cols, perm, int(total.item())


def _matrix(M, K, sparsity, seed):
    import sparsecore_b200 as sl

    g = torch.Generator().manual_seed(seed)
    mask = torch.rand(M, K, generator=g) >= sparsity
    dense = torch.randn(M, K, generator=g) * mask
    return sl.PaddedCSR.from_dense(dense.cuda())


@pytest.mark.parametrize("opp", [1.2, 1.0])
def test_noalloc_transpose_matches_allocating_path_twice(opp):
    cases = [(300, 517, 0.9, 1), (97, 1030, 0.5, 2)]
    for M, K, s, seed in cases:  # two calls in a row on the shared scratch
        W = _matrix(M, K, s, seed)
        WT, perm_ref = _reference_transpose(W, opp)
        rows, vals, cols, perm, total = _noalloc_transpose(W, opp)
        assert total == WT.total_capacity
        assert torch.equal(rows[0], WT.row_nnz)
        assert torch.equal(rows[1], WT.row_capacity)
        assert torch.equal(rows[2], WT.row_start)
        assert torch.equal(cols[:total], WT.col_indices)
        assert torch.equal(vals[:total].view(torch.int32), WT.values.view(torch.int32))
        assert torch.equal(perm[:total], perm_ref)
        # entries past the true size are padding
        assert bool((cols[total:] == -1).all()) and bool((perm[total:] == -1).all())
        assert bool((vals[total:] == 0).all())


def test_noalloc_transpose_rejects_oversize_and_short_buffers():
    from sparsecore_b200 import _native as N

    lib = N.lib()
    # ceil(nrows/32) * ncols beyond the 2^20 static counters -> SL_ERR_UNSUPPORTED
    big = N.SlCsr(32 * 64, 20000, 0, None, None, 1, 1, 1)
    WT = N.SlCsr(20000, 32 * 64, 1 << 20, 1, 1, 1, 1, 1)
    rc = lib.sl_transpose_with_perm_noalloc(ctypes.byref(big), 1.2, ctypes.byref(WT), N.P(1),
                                            N.P(1), N.P(0))
    assert rc == N.SL_ERR_UNSUPPORTED
    assert b"static scratch" in lib.sl_last_error()
    # slot arrays shorter than the documented bound -> SL_ERR_INVALID
    W = _matrix(64, 64, 0.8, 3)
    short = N.SlCsr(64, 64, 10, 1, 1, 1, 1, 1)
    rc = lib.sl_transpose_with_perm_noalloc(W._abi_ref(), 1.2, ctypes.byref(short), N.P(1),
                                            N.P(1), W._stream())
    assert rc == N.SL_ERR_INVALID
    assert b"required" in lib.sl_last_error()


_FIRST_CALL_SCRIPT = r"""
import ctypes, math, sys
import numpy as np
import torch
sys.path.insert(0, sys.argv[1])
from sparsecore_b200 import _native as N

# A padded CSR built with numpy and plain copies: no library kernel runs
# before the allocation-free entry point.
rng = np.random.default_rng(5)
M, K, opp = 200, 333, 1.2
mask = rng.random((M, K)) >= 0.85
nnz = mask.sum(1).astype(np.int32)
cap = np.maximum(1, np.ceil(nnz * opp)).astype(np.int32)
rs = np.concatenate([[0], np.cumsum(cap)[:-1]]).astype(np.int32)
tot = int(cap.sum())
vals = np.zeros(tot, np.float32); cols = np.full(tot, -1, np.int32)
for i in range(M):
    c = np.nonzero(mask[i])[0]
    cols[rs[i]:rs[i] + len(c)] = c
    vals[rs[i]:rs[i] + len(c)] = rng.standard_normal(len(c)).astype(np.float32)
d = torch.device("cuda", 0)
t = {k: torch.from_numpy(v).to(d) for k, v in
     dict(vals=vals, cols=cols, rs=rs, nnz=nnz, cap=cap).items()}
W = N.SlCsr(M, K, tot, t["vals"].data_ptr(), t["cols"].data_ptr(), t["rs"].data_ptr(),
            t["nnz"].data_ptr(), t["cap"].data_ptr())
bound = int(math.floor(opp * tot)) + K + 2
rows = torch.empty(3, K, dtype=torch.int32, device=d)
wv = torch.empty(bound, dtype=torch.float32, device=d)
wc = torch.empty(bound, dtype=torch.int32, device=d)
perm = torch.empty(bound, dtype=torch.int64, device=d)
total = torch.zeros(1, dtype=torch.int64, device=d)
WT = N.SlCsr(K, M, bound, wv.data_ptr(), wc.data_ptr(), rows[2].data_ptr(), rows[0].data_ptr(),
             rows[1].data_ptr())
N.check(N.lib().sl_transpose_with_perm_noalloc(ctypes.byref(W), opp, ctypes.byref(WT),
                                               N.ptr(perm), N.ptr(total), None))
torch.cuda.synchronize()
n = int(total.item())

import sparsecore_b200 as sl
P = sl.PaddedCSR(M, K, vals, cols, rs, nnz, cap, device=d)
RT, rperm = sl.transpose_with_perm(P, padding_ratio=opp - 1.0)
ok = (n == RT.total_capacity and torch.equal(rows[0], RT.row_nnz)
      and torch.equal(rows[1], RT.row_capacity) and torch.equal(rows[2], RT.row_start)
      and torch.equal(wc[:n], RT.col_indices) and torch.equal(perm[:n], rperm)
      and torch.equal(wv[:n].view(torch.int32), RT.values.view(torch.int32)))
print("FIRST_CALL_OK" if ok else "FIRST_CALL_MISMATCH")
"""


def test_noalloc_transpose_as_first_library_call_in_a_fresh_process():
    """The first call on a device also looks up the scratch array's address
    (and, with lazy module loading, makes CUDA load the library's device
    code): run it before any other kernel of the library in a new process."""
    import os
    import subprocess
    import sys

    repo = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    out = subprocess.run([sys.executable, "-c", _FIRST_CALL_SCRIPT, repo], capture_output=True,
                         text=True, timeout=600)
    assert "FIRST_CALL_OK" in out.stdout, out.stdout + out.stderr
