"""Router state round trip of the checkpoint module (host only)."""
import numpy as np
import pytest


def test_router_state_roundtrip_continues_the_draws():
    import sparsecore_b200 as sl
    from sparsecore_b200.checkpoint import load_router_state, router_state

    a = sl.SET(sparsity=0.9, seed=3)
    a._step_idx = 41
    a._rng.choice(50, size=7, replace=False)
    st = router_state(a)
    expected = a._rng.choice(100, size=9, replace=False)
    b = sl.SET(sparsity=0.9, seed=999)
    load_router_state(b, st)
    assert b._step_idx == 41
    assert np.array_equal(b._rng.choice(100, size=9, replace=False), expected)
    with pytest.raises(ValueError):
        load_router_state(sl.RigL(sparsity=0.9), st)
