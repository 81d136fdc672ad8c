"""Pin the CPU oracle against golden vectors produced by the reference itself
(tests/golden/make_golden.py).  CPU only."""
import numpy as np
import pytest

from oracle import oracle as O


def bits_equal(a, b):
    a = np.ascontiguousarray(a, np.float32)
    b = np.ascontiguousarray(b, np.float32)
    return a.shape == b.shape and np.array_equal(a.view(np.int32), b.view(np.int32))


def csr_equal(p, q):
    return (p.nrows == q.nrows and p.ncols == q.ncols and bits_equal(p.values, q.values)
            and np.array_equal(p.cols, q.cols) and np.array_equal(p.row_start, q.row_start)
            and np.array_equal(p.row_nnz, q.row_nnz)
            and np.array_equal(p.row_capacity, q.row_capacity))


def kernel_ids(golden):
    return range(len(golden.meta["kernel_cases"]))


@pytest.mark.parametrize("idx", range(12))
def test_oracle_kernels_match_reference(golden, idx):
    p = f"k{idx}_"
    W = golden.csr(p + "W_")
    X, dY = golden[p + "X"], golden[p + "dY"]
    assert O.check_invariants(W)[0] == 0
    # forward: bit-exact FMA chain in slot order
    assert bits_equal(O.spmm(W, X), golden[p + "Y"])
    # dW: bit-exact AVX2 lane order
    assert bits_equal(O.sddmm(W, dY, X), golden[p + "dW"])
    # transpose + perm: bit-exact arrays
    WT, perm = O.transpose_with_perm(W)
    assert csr_equal(WT, golden.csr(p + "WT_"))
    assert np.array_equal(perm, golden[p + "perm"])
    # dX over the transpose: bit-exact
    assert bits_equal(O.spmm(WT, dY), golden[p + "dX"])
    # dense gradient: bit-exact with the reference build's in-order
    # vectorised reduction (rounded products, FMA for the last N mod 4)
    assert bits_equal(O.dense_grad(dY, X), golden[p + "G"])


def test_oracle_capacity_and_from_dense():
    rn = np.array([0, 1, 4, 5, 10, 13, 100, 7], np.int32)
    assert list(O.capacity(rn, 0.2)) == [1, 2, 5, 6, 12, 16, 120, 9]
    assert list(O.capacity(rn, 0.0)) == [1, 1, 4, 5, 10, 13, 100, 7]
    with pytest.raises(ValueError):
        O.capacity(rn, -0.1)
    rng = np.random.default_rng(0)
    D = rng.standard_normal((20, 30)).astype(np.float32)
    D[rng.random(D.shape) < 0.8] = 0
    p = O.from_dense(D)
    assert O.check_invariants(p)[0] == 0
    assert np.array_equal(O.to_dense(p), D)


def test_oracle_invariant_codes():
    p = O.from_dense(np.eye(4, dtype=np.float32))
    q = p.copy(); q.row_start[2] += 1
    assert O.check_invariants(q)[:2] == (3, 2)
    q = p.copy(); q.row_nnz[1] = 5
    assert O.check_invariants(q)[:2] == (4, 1)
    q = p.copy(); q.cols[q.row_start[3]] = 9
    assert O.check_invariants(q) == (6, 3, 0)
    q = p.copy(); q.cols[q.row_start[0] + 1] = 2
    assert O.check_invariants(q) == (7, 0, 1)


@pytest.mark.parametrize("idx", range(7))
def test_oracle_set_matches_reference(golden, idx):
    fin, fout, s, df, seed, tie, nup = golden.meta["set_cases"][idx]
    p = f"set{idx}_"
    W = golden.csr(p + "in_")
    rng = np.random.default_rng(seed)
    for u in range(nup):
        O.set_update(W, df, rng)
        assert csr_equal(W, golden.csr(f"{p}out{u}_")), f"update {u}"
        W = golden.csr(f"{p}pert{u}_")


@pytest.mark.parametrize("idx", range(5))
def test_oracle_rigl_matches_reference(golden, idx):
    fin, fout, s, df, kind = golden.meta["rigl_cases"][idx]
    p = f"rigl{idx}_"
    W = golden.csr(p + "in_")
    O.rigl_update(W, df, golden[p + "G"])
    assert csr_equal(W, golden.csr(p + "out_"))
