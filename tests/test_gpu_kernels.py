"""GPU parity: forward SpMM, SDDMM dW, transpose + dX and dense_grad against
the reference's golden outputs (bit-exact), through the C-ABI library."""
import numpy as np
import pytest
import torch

from gpu_helpers import bits_equal, csr_from_golden, csr_matches, dev, host, oracle_csr, sha

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("idx", range(12))
def test_kernels_bit_exact_vs_reference(golden, idx):
    import sparsecore_b200 as sl
    from sparsecore_b200 import ops

    p = f"k{idx}_"
    W = csr_from_golden(golden, p + "W_")
    X = torch.from_numpy(golden[p + "X"]).to(dev())
    dY = torch.from_numpy(golden[p + "dY"]).to(dev())
    assert bits_equal(sl.spmm(W, X), golden[p + "Y"])
    assert bits_equal(ops._sddmm_raw(W, dY, X), golden[p + "dW"])
    WT, perm = sl.transpose_with_perm(W)
    assert csr_matches(WT, golden, p + "WT_")
    assert np.array_equal(host(perm), golden[p + "perm"])
    assert bits_equal(ops._spmm_raw(WT, dY), golden[p + "dX"])
    assert bits_equal(sl.dense_grad(dY, X), golden[p + "G"])


@pytest.mark.parametrize("idx", [0, 3, 6, 10])
def test_autograd_matches_reference(golden, idx):
    import sparsecore_b200 as sl
    from sparsecore_b200.ops import _clear_transpose_cache

    _clear_transpose_cache()
    p = f"k{idx}_"
    W = csr_from_golden(golden, p + "W_")
    X = torch.from_numpy(golden[p + "X"]).to(dev()).requires_grad_(True)
    dY = torch.from_numpy(golden[p + "dY"]).to(dev())
    Wv = torch.nn.Parameter(W.values)
    from sparsecore_b200.ops import _SpMMFunction

    Y = _SpMMFunction.apply(Wv, W, X, "simd")
    Y.backward(dY)
    assert bits_equal(Y, golden[p + "Y"])
    assert bits_equal(Wv.grad, golden[p + "dW"])
    assert bits_equal(X.grad, golden[p + "dX"])
    # the Parameter aliases the CSR storage
    assert Wv.data_ptr() == W.values.data_ptr()


def test_random_factory_matches_reference(golden):
    import sparsecore_b200 as sl

    for idx, (M, K, N, s, seed) in enumerate(golden.meta["kernel_cases"]):
        W = sl.PaddedCSR.random(M, K, sparsity=s, seed=seed)
        assert csr_matches(W, golden, f"k{idx}_W_"), idx


def test_config1_sparse_linear_bit_exact(golden):
    """cfg1: SparseLinear(784,256,90%) init + Y/dW/dX vs reference hashes."""
    import sparsecore_b200 as sl
    from sparsecore_b200 import ops

    m = golden.meta["cfg1"]
    torch.manual_seed(0)
    layer = sl.SparseLinear(784, 256, sparsity=0.9, bias=False)
    W = layer._csr
    assert W.nnz == m["nnz"] and W.total_capacity == m["total_capacity"]
    assert sha(host(W.values)) == m["sha_values"]
    assert sha(host(W.col_indices)) == m["sha_cols"]
    g = torch.Generator().manual_seed(1)
    X = torch.randn(784, 256, generator=g)
    dY = torch.randn(256, 256, generator=g)
    assert sha(X.numpy()) == m["sha_X"] and sha(dY.numpy()) == m["sha_dY"]
    X, dY = X.to(dev()), dY.to(dev())
    assert sha(host(sl.spmm(W, X))) == m["sha_Y"]
    assert sha(host(ops._sddmm_raw(W, dY, X))) == m["sha_dW"]
    WT, perm = sl.transpose_with_perm(W)
    assert sha(host(WT.col_indices)) == m["sha_WT_cols"]
    assert sha(host(perm)) == m["sha_perm"]
    assert sha(host(ops._spmm_raw(WT, dY))) == m["sha_dX"]


@pytest.mark.parametrize("M,K,N,s", [(4096, 4096, 32, 0.9), (4096, 4096, 256, 0.9),
                                     (16384, 4096, 1, 0.5), (2048, 4096, 257, 0.99),
                                     (1024, 3072, 96, 0.9)])
def test_config3_shapes_vs_oracle(M, K, N, s):
    """Standalone SpMM sweep shapes: GPU vs the C oracle, bit-exact."""
    import sparsecore_b200 as sl
    from oracle import oracle as O
    from sparsecore_b200 import ops

    g = torch.Generator().manual_seed(M + N)
    mask = torch.rand(M, K, generator=g) < (1 - s)
    Wd = torch.randn(M, K, generator=g) * 0.02 * mask
    W = sl.PaddedCSR.from_dense(Wd.to(dev()))
    X = torch.randn(K, N, generator=g)
    dY = torch.randn(M, N, generator=g)
    Xd, dYd = X.to(dev()), dY.to(dev())
    Wo = oracle_csr(W)
    assert bits_equal(sl.spmm(W, Xd), O.spmm(Wo, X.numpy()))
    assert bits_equal(ops._sddmm_raw(W, dYd, Xd), O.sddmm(Wo, dY.numpy(), X.numpy()))
    WT, perm = sl.transpose_with_perm(W)
    WTo, permo = O.transpose_with_perm(Wo)
    assert np.array_equal(host(WT.col_indices), WTo.cols)
    assert np.array_equal(host(perm), permo)
    assert bits_equal(ops._spmm_raw(WT, dYd), O.spmm(WTo, dY.numpy()))


def test_edge_cases():
    import sparsecore_b200 as sl
    from oracle import oracle as O
    from sparsecore_b200 import ops

    d = dev()
    # empty rows, one dense row, N=1 / N=5 (unaligned vectors), unaligned base pointer
    Wd = torch.zeros(9, 13)
    Wd[2, 3] = 1.5
    Wd[4] = torch.arange(13, dtype=torch.float32) - 6
    Wd[7, 12] = -2.0
    W = sl.PaddedCSR.from_dense(Wd.to(d))
    assert W.nnz == 1 + 12 + 1
    Wo = oracle_csr(W)
    for N in (1, 2, 5, 16, 17, 31, 64, 129):
        X = torch.randn(13, N)
        dY = torch.randn(9, N)
        assert bits_equal(sl.spmm(W, X.to(d)), O.spmm(Wo, X.numpy()))
        assert bits_equal(ops._sddmm_raw(W, dY.to(d), X.to(d)), O.sddmm(Wo, dY.numpy(), X.numpy()))
        # base pointer offset by one float -> not 16-byte aligned
        buf = torch.empty(13 * N + 1, device=d)
        Xu = buf[1:].view(13, N)
        Xu.copy_(X)
        assert bits_equal(sl.spmm(W, Xu), O.spmm(Wo, X.numpy()))
    # all-zero matrix, zero-capacity matrix, N = 0
    Z = sl.PaddedCSR.from_dense(torch.zeros(5, 7, device=d))
    assert Z.nnz == 0 and Z.total_capacity == 5
    assert torch.count_nonzero(sl.spmm(Z, torch.randn(7, 3, device=d))) == 0
    E = sl.PaddedCSR(4, 6)
    assert E.total_capacity == 0
    assert torch.count_nonzero(sl.spmm(E, torch.randn(6, 4, device=d))) == 0
    assert sl.spmm(W, torch.randn(13, 0, device=d)).shape == (9, 0)
    # transpose of an empty / zero-capacity matrix
    ET = sl.PaddedCSR.transpose(E)
    assert ET.shape == (6, 4) and ET.nnz == 0 and ET.total_capacity == 6


def test_transpose_involution_and_padding_ratio():
    import sparsecore_b200 as sl

    W = sl.PaddedCSR.random(300, 200, sparsity=0.9, seed=3)
    WT = W.transpose()
    WTT = WT.transpose()
    assert torch.equal(WTT.to_dense(), W.to_dense())
    assert torch.equal(WT.to_dense(), W.to_dense().t())
    W0 = W.transpose(padding_ratio=0.0)
    assert W0.padding_slots == int((host(W0.row_nnz) == 0).sum())
    with pytest.raises(ValueError):
        W.transpose(padding_ratio=-1.0)


@pytest.mark.parametrize("pack", ["1", "0"])
@pytest.mark.parametrize("path", ["rows", "xs", "xs32", "xs64"])
def test_forward_paths_and_sddmm_variants_vs_oracle(path, pack, monkeypatch):
    """Both forward decompositions (row-gather and X-stationary with 128-,
    64- and 32-column tiles, with packed 16-bit-column or pair staging), the
    lane and quad SDDMM kernels, ragged row lengths (one dense row among
    sparse ones, empty rows) and column counts around every dispatch
    threshold (partial last tiles included)."""
    import sparsecore_b200 as sl
    from oracle import oracle as O
    from sparsecore_b200 import ops

    if path == "rows" and pack == "0":
        pytest.skip("staging form applies to the X-stationary kernel only")
    monkeypatch.setenv("SPARSECORE_B200_XS_PACK", pack)
    monkeypatch.setenv("SPARSECORE_B200_FWD", "xs" if path.startswith("xs") else path)
    if path in ("xs32", "xs64"):  # default: the widest tile that fits (here 64 for W, 128 for W^T)
        monkeypatch.setenv("SPARSECORE_B200_XS_TN", path[2:])
    d = dev()
    g = torch.Generator().manual_seed(11)
    M, K = 301, 517
    mask = torch.rand(M, K, generator=g) < 0.1
    mask[7] = True          # one dense row: several segments per warp pass
    mask[100:140] = False   # empty rows
    Wd = torch.randn(M, K, generator=g) * mask
    W = sl.PaddedCSR.from_dense(Wd.to(d))
    Wo = oracle_csr(W)
    WT, _ = sl.transpose_with_perm(W)
    WTo, _ = O.transpose_with_perm(Wo)
    for N in (1, 3, 4, 8, 12, 20, 36, 63, 64, 68, 252, 256, 260, 384, 1000):
        X = torch.randn(K, N, generator=g)
        dY = torch.randn(M, N, generator=g)
        Xd, dYd = X.to(d), dY.to(d)
        assert bits_equal(sl.spmm(W, Xd), O.spmm(Wo, X.numpy())), N
        assert bits_equal(ops._sddmm_raw(W, dYd, Xd), O.sddmm(Wo, dY.numpy(), X.numpy())), N
        assert bits_equal(ops._spmm_raw(WT, dYd), O.spmm(WTo, dY.numpy())), N


@pytest.mark.parametrize("M,K,N,block", [(301, 517, 256, False), (700, 300, 512, True),
                                         (96, 2000, 288, False), (1000, 1000, 320, True),
                                         (2100, 3100, 256, True)])
def test_mid_n_sddmm_and_forward_vs_oracle(M, K, N, block, monkeypatch):
    """N = 256-512, below the tiled SDDMM's N >= 1024 threshold: the quad
    SDDMM kernel (the tile-order knob has no effect here, so all three
    launches below run it) and the forward / dX kernels against the oracle,
    with edge rows and a dense block.  The tiled kernel's own parity cases
    are in test_gpu_sddmm_tiled.py."""
    import sparsecore_b200 as sl
    from oracle import oracle as O
    from sparsecore_b200 import ops

    d = dev()
    g = torch.Generator().manual_seed(M + K)
    mask = torch.rand(M, K, generator=g) < 0.06
    if block:
        mask[:130, :70] = True
    Wd = torch.randn(M, K, generator=g) * mask
    W = sl.PaddedCSR.from_dense(Wd.to(d))
    X = torch.randn(K, N, generator=g)
    dY = torch.randn(M, N, generator=g)
    Wo = oracle_csr(W)
    # forward on the same shapes (K > 1536 runs the row-gather kernel)
    assert bits_equal(sl.spmm(W, X.to(d)), O.spmm(Wo, X.numpy()))
    WT, _ = sl.transpose_with_perm(W)
    WTo, _ = O.transpose_with_perm(Wo)
    assert bits_equal(ops._spmm_raw(WT, dY.to(d)), O.spmm(WTo, dY.numpy()))
    dw = ops._sddmm_raw(W, dY.to(d), X.to(d))
    other = "row" if K > M else "col"  # the tile order the default did not take
    monkeypatch.setenv("SPARSECORE_B200_DW_ORDER", other)
    dw_other_order = ops._sddmm_raw(W, dY.to(d), X.to(d))
    monkeypatch.setenv("SPARSECORE_B200_DW", "quad")
    per_slot = ops._sddmm_raw(W, dY.to(d), X.to(d))
    assert bits_equal(dw, per_slot)
    assert bits_equal(dw_other_order, per_slot)
    assert bits_equal(dw, O.sddmm(Wo, dY.numpy(), X.numpy()))


@pytest.mark.parametrize("M,K,s,pr", [(70, 50, 0.5, 0.2), (9, 13, 0.0, 0.0), (129, 20000, 0.995, 0.2),
                                      (300, 3000, 0.9, 0.0), (1000, 700, 0.97, 0.2),
                                      (12000, 300, 0.9, 0.0), (7, 5, 0.3, 0.0), (4733, 1001, 0.8, 0.0),
                                      (300, 17000, 0.9, 0.2)])
def test_spmv_lane_kernel_matches_oracle_and_warp_kernel(M, K, s, pr, monkeypatch):
    """N = 1: forward / dX on the lane-per-row kernels (warp-specialised row
    windows by default, both ring depths, X staged or through L1; the per-lane
    cp.async variant) and the
    streaming SDDMM, against the oracle and the general kernels: ragged and
    empty rows, rows whose 4-slot groups start unaligned or run past the
    arrays' end (no padding, total capacity not a multiple of 4), K above
    the shared-memory X limit, one long row among short ones, and more rows
    than one or two warps per SM (the other configurations)."""
    import sparsecore_b200 as sl
    from oracle import oracle as O
    from sparsecore_b200 import ops

    d = dev()
    g = torch.Generator().manual_seed(M * 7 + K)
    mask = torch.rand(M, K, generator=g) >= s
    mask[min(3, M - 1)] = False  # an empty row
    mask[M // 2, : min(K, 2500)] = True  # a long row
    Wd = torch.randn(M, K, generator=g) * mask
    W = sl.PaddedCSR.from_dense(Wd.to(d), padding_ratio=pr)
    Wo = oracle_csr(W)
    X = torch.randn(K, 1, generator=g)
    dY = torch.randn(M, 1, generator=g)
    WT, _ = sl.transpose_with_perm(W)
    WTo, _ = O.transpose_with_perm(Wo)
    y = sl.spmm(W, X.to(d))
    dx = ops._spmm_raw(WT, dY.to(d))
    dw = ops._sddmm_raw(W, dY.to(d), X.to(d))  # streaming N = 1 SDDMM
    assert bits_equal(y, O.spmm(Wo, X.numpy()))
    assert bits_equal(dx, O.spmm(WTo, dY.numpy()))
    assert bits_equal(dw, O.sddmm(Wo, dY.numpy(), X.numpy()))
    monkeypatch.setenv("SPARSECORE_B200_N1", "ws")  # forced: short rows default to the lane kernel
    for xs in ("1", "0"):  # X in shared memory / through L1
        monkeypatch.setenv("SPARSECORE_B200_N1_XS", xs)
        for st in ("4", "8"):  # both ring depths
            for rpc in ("16", "32"):  # rows per CTA
                monkeypatch.setenv("SPARSECORE_B200_N1_ST", st)
                monkeypatch.setenv("SPARSECORE_B200_N1_RPC", rpc)
                assert bits_equal(sl.spmm(W, X.to(d)), y), (xs, st, rpc)
                assert bits_equal(ops._spmm_raw(WT, dY.to(d)), dx), (xs, st, rpc)
    monkeypatch.delenv("SPARSECORE_B200_N1_RPC")
    monkeypatch.delenv("SPARSECORE_B200_N1_ST")
    monkeypatch.delenv("SPARSECORE_B200_N1_XS")
    monkeypatch.setenv("SPARSECORE_B200_N1", "lane")  # the cp.async lane kernel
    assert bits_equal(sl.spmm(W, X.to(d)), y)
    assert bits_equal(ops._spmm_raw(WT, dY.to(d)), dx)
    monkeypatch.setenv("SPARSECORE_B200_N1", "warp")
    assert bits_equal(sl.spmm(W, X.to(d)), y)
    assert bits_equal(ops._spmm_raw(WT, dY.to(d)), dx)
    assert bits_equal(ops._sddmm_raw(W, dY.to(d), X.to(d)), dw)


@pytest.mark.parametrize("M,K,s,pr", [(70, 50, 0.5, 0.2), (9, 13, 0.0, 0.0), (300, 3000, 0.9, 0.0),
                                      (1000, 700, 0.97, 0.2), (2000, 300, 0.8, 0.2)])
def test_lanerow_small_n_matches_oracle_and_warp_kernel(M, K, s, pr, monkeypatch):
    """N = 4 and 8: forward / dX on the lane-per-row kernel (one lane per
    row, N column chains per lane; forced here, by default it runs only with
    many rows) against the oracle and the warp-per-row kernel: ragged and empty rows, no padding (the last group
    read past the arrays' end), one long row among short ones."""
    import sparsecore_b200 as sl
    from oracle import oracle as O
    from sparsecore_b200 import ops

    d = dev()
    g = torch.Generator().manual_seed(M * 5 + K)
    mask = torch.rand(M, K, generator=g) >= s
    mask[min(3, M - 1)] = False
    mask[M // 2, : min(K, 2500)] = True
    W = sl.PaddedCSR.from_dense((torch.randn(M, K, generator=g) * mask).to(d), padding_ratio=pr)
    Wo = oracle_csr(W)
    WT, _ = sl.transpose_with_perm(W)
    WTo, _ = O.transpose_with_perm(Wo)
    for N in (4, 8):
        X = torch.randn(K, N, generator=g)
        dY = torch.randn(M, N, generator=g)
        monkeypatch.setenv("SPARSECORE_B200_SMALLN", "lane")
        y = sl.spmm(W, X.to(d))
        dx = ops._spmm_raw(WT, dY.to(d))
        assert bits_equal(y, O.spmm(Wo, X.numpy())), N
        assert bits_equal(dx, O.spmm(WTo, dY.numpy())), N
        monkeypatch.setenv("SPARSECORE_B200_SMALLN", "warp")
        assert bits_equal(sl.spmm(W, X.to(d)), y), N
        assert bits_equal(ops._spmm_raw(WT, dY.to(d)), dx), N
        monkeypatch.delenv("SPARSECORE_B200_SMALLN")


@pytest.mark.parametrize("M,K,s", [(301, 517, 0.9), (2000, 4096, 0.95), (50, 70, 0.0)])
def test_n32_gather_kernels_vs_oracle(M, K, s, monkeypatch):
    """N = 32: the SDDMM (default) and forward (forced) kernels that stage X
    rows by cp.async, and the row-warp forward, against the oracle and each
    other: empty rows, rows of
    exactly 32 / 33 / 64 slots (chunk edges) and one long row, so the
    register ring and the staging ring both wrap."""
    import sparsecore_b200 as sl
    from oracle import oracle as O
    from sparsecore_b200 import ops

    from gpu_helpers import launched_kernels

    d = dev()
    g = torch.Generator().manual_seed(M + K)
    mask = torch.rand(M, K, generator=g) >= s
    mask[1] = False
    if M > 10:
        for r, n in ((2, 32), (3, 33), (4, 64), (5, 31)):
            mask[r] = False
            mask[r, :n] = True
        mask[M // 2] = True  # a long row: many chunks
    W = sl.PaddedCSR.from_dense((torch.randn(M, K, generator=g) * mask).to(d))
    Wo = oracle_csr(W)
    WT, _ = sl.transpose_with_perm(W)
    WTo, _ = O.transpose_with_perm(Wo)
    X = torch.randn(K, 32, generator=g)
    dY = torch.randn(M, 32, generator=g)
    y, names = launched_kernels(lambda: sl.spmm(W, X.to(d)))
    assert names == ["spmm_rowwarp_kernel"], names  # the N = 32 forward default
    monkeypatch.setenv("SPARSECORE_B200_N32", "gather")
    y_staged, names = launched_kernels(lambda: sl.spmm(W, X.to(d)))
    assert names == ["gather32_fwd_kernel"], names
    assert bits_equal(y_staged, y)
    monkeypatch.delenv("SPARSECORE_B200_N32")
    dw, names = launched_kernels(lambda: ops._sddmm_raw(W, dY.to(d), X.to(d)))
    assert names == ["gather32_sddmm_kernel"], names
    dx = ops._spmm_raw(WT, dY.to(d))
    assert bits_equal(y, O.spmm(Wo, X.numpy()))
    assert bits_equal(dw, O.sddmm(Wo, dY.numpy(), X.numpy()))
    assert bits_equal(dx, O.spmm(WTo, dY.numpy()))
    monkeypatch.setenv("SPARSECORE_B200_N32", "rows")
    assert bits_equal(sl.spmm(W, X.to(d)), y)
    assert bits_equal(ops._sddmm_raw(W, dY.to(d), X.to(d)), dw)


@pytest.mark.parametrize("M,K,N", [(300, 517, 1001), (1536, 384, 2048), (130, 129, 7)])
def test_dense_grad_both_tilings_vs_oracle(M, K, N, monkeypatch):
    """RigL's dense gradient on the 64x64 and the 128x128 (double-buffered)
    GEMM tilings: ragged edges, N not a multiple of 4 (the FMA tail), bit-exact
    against the oracle's restatement of the reference loop."""
    import sparsecore_b200 as sl
    from oracle import oracle as O

    g = torch.Generator().manual_seed(M + K + N)
    dY = torch.randn(M, N, generator=g)
    X = torch.randn(K, N, generator=g)
    ref = O.dense_grad(dY.numpy(), X.numpy())
    for tiling in ("64", "128"):
        monkeypatch.setenv("SPARSECORE_B200_DG", tiling)
        assert bits_equal(sl.dense_grad(dY.to(dev()), X.to(dev())), ref), tiling
