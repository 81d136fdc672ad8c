"""LiveAdamW (fused AdamW over live slots, sl_adamw_live) against
torch.optim.AdamW on the same model and data: equal to float rounding over
several steps and across a SET topology update (per-slot state stays with
the slot in both), padding slots stay exactly zero, and the dense
parameters follow torch's AdamW (to the same tolerance: their gradients
see the sparse weights' rounding differences)."""
import pytest
import torch

from gpu_helpers import dev

pytestmark = pytest.mark.gpu


def _model():
    import sparsecore_b200 as sl

    torch.manual_seed(3)
    return torch.nn.Sequential(sl.SparseLinear(96, 64, sparsity=0.8, device=dev()), torch.nn.GELU(),
                               sl.SparseLinear(64, 32, sparsity=0.9, device=dev()),
                               torch.nn.Linear(32, 8).to(dev()))


def test_live_adamw_matches_torch_adamw_across_a_topology_update():
    import sparsecore_b200 as sl
    from sparsecore_b200.optim import LiveAdamW

    a, b = _model(), _model()  # same seed: identical weights and masks
    opt_a = torch.optim.AdamW(a.parameters(), lr=3e-3, weight_decay=0.01)
    opt_b = LiveAdamW(b, lr=3e-3, weight_decay=0.01)
    algo_a = sl.SET(0.8, drop_fraction=0.3, update_freq=4, seed=1)
    algo_b = sl.SET(0.8, drop_fraction=0.3, update_freq=4, seed=1)
    a.apply(algo_a)
    b.apply(algo_b)
    g = torch.Generator().manual_seed(0)
    for step in range(9):
        x = torch.randn(40, 96, generator=g).to(dev())
        for model, opt, algo in ((a, opt_a, algo_a), (b, opt_b, algo_b)):
            opt.zero_grad(set_to_none=True)
            model(x).square().mean().backward()
            opt.step()
            algo.step()
        for m_a, m_b in zip(a, b):
            if isinstance(m_a, sl.SparseLinear):
                assert torch.equal(m_a._csr.col_indices, m_b._csr.col_indices), step
                torch.testing.assert_close(m_b._values, m_a._values, rtol=1e-5, atol=1e-7)
                pad = m_b._csr.col_indices < 0
                assert bool((m_b._values[pad] == 0).all())
    # the dense layer follows torch's AdamW; its gradients see the sparse
    # weights' rounding differences, so it agrees to the same tolerance
    torch.testing.assert_close(b[3].weight, a[3].weight, rtol=1e-5, atol=1e-7)
    assert algo_b._step_idx == 9 and algo_b.last_update_step == 8


def test_live_adamw_rejects_bad_hyper_parameters():
    from sparsecore_b200.optim import LiveAdamW

    with pytest.raises(ValueError):
        LiveAdamW(_model(), lr=-1.0)
