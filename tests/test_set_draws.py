"""SET regrow draws in the native library against numpy itself: the ranks
and the generator state after the draws equal the reference's per-row loop
of ``rng.choice(pool, size=n_grow, replace=False)`` (sparselab/router.py:
457-470) on an identical Generator(PCG64), including a pending 32-bit half
in the generator state and pools above 10000 (numpy's tail-shuffle path).
Host-only: runs without a GPU."""
import numpy as np
import pytest

from sparsecore_b200 import _native as N


@pytest.fixture(scope="module", autouse=True)
def lib():
    from sparsecore_b200.build import build

    build()
    N._lib = N.load_library()
    yield
    N._lib = None


def _reference_loop(rng, n_live, n_keep, ncols):
    counts = np.zeros(len(n_live), np.int32)
    draws = []
    for i in np.nonzero(n_live)[0]:
        nk = int(n_keep[i])
        n_drop, pool = int(n_live[i]) - nk, ncols - nk
        if pool == 0 or n_drop == 0:
            continue
        n_grow = min(n_drop, pool)
        draws.append(rng.choice(pool, size=n_grow, replace=False))
        counts[i] = n_grow
    return counts, (np.concatenate(draws).astype(np.int32) if draws else np.zeros(0, np.int32))


@pytest.mark.parametrize("seed", range(6))
@pytest.mark.parametrize("ncols,density,pending32", [(50, 0.3, False), (768, 0.1, True), (3072, 0.1, False),
                                                      (12000, 0.2, False), (30000, 0.05, True), (7, 1.0, False)])
def test_native_draws_match_numpy(seed, ncols, density, pending32):
    from sparsecore_b200.router import _regrow_draws

    g = np.random.default_rng(1000 + seed)
    nrows = 40
    n_live = (g.random(nrows) * 2 * density * ncols).astype(np.int32).clip(0, ncols)
    n_live[::7] = 0
    n_keep = (n_live * g.uniform(0.3, 1.0, nrows)).astype(np.int32)
    n_keep[3] = n_live[3]  # nothing dropped
    a, b = np.random.default_rng(seed), np.random.default_rng(seed)
    if pending32:  # leave half of a 64-bit output buffered in the state
        a.integers(0, 1000, dtype=np.int32)
        b.integers(0, 1000, dtype=np.int32)
        assert a.bit_generator.state["has_uint32"] == 1
    want_c, want_r = _reference_loop(a, n_live, n_keep, ncols)
    got_c, got_r = _regrow_draws(b, n_live, n_keep, ncols)
    assert np.array_equal(got_c, want_c)
    assert np.array_equal(got_r, want_r)
    assert b.bit_generator.state == a.bit_generator.state
    assert b.random() == a.random()  # and the streams continue identically


def test_tail_shuffle_path_is_taken_and_matches():
    from sparsecore_b200.router import _regrow_draws

    # pool = 20000 > 10000 and n_grow = 5000 > pool / 50: numpy's tail shuffle
    n_live, n_keep = np.array([5000], np.int32), np.array([0], np.int32)
    a, b = np.random.default_rng(7), np.random.default_rng(7)
    want = a.choice(20000, size=5000, replace=False)
    _, got = _regrow_draws(b, n_live, n_keep, 20000)
    assert np.array_equal(got, want.astype(np.int32))
    assert b.bit_generator.state == a.bit_generator.state


def test_non_pcg64_generator_takes_the_per_row_loop():
    from sparsecore_b200.router import _regrow_draws

    n_live = np.array([10, 0, 7, 5], np.int32)
    n_keep = np.array([6, 0, 7, 1], np.int32)
    a = np.random.Generator(np.random.MT19937(3))
    b = np.random.Generator(np.random.MT19937(3))
    want = _reference_loop(a, n_live, n_keep, 40)
    got = _regrow_draws(b, n_live, n_keep, 40)
    assert np.array_equal(got[0], want[0]) and np.array_equal(got[1], want[1])
    assert b.random() == a.random()
