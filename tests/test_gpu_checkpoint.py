"""Checkpoints with topology: a run resumed from a checkpoint taken between
SET updates continues bit-identically (masks, values, optimizer moments,
future random draws), also into a model built from a different seed."""
import numpy as np
import pytest
import torch

from gpu_helpers import dev

pytestmark = pytest.mark.gpu


def _make(seed):
    import sparsecore_b200 as sl

    torch.manual_seed(seed)
    model = torch.nn.Sequential(sl.SparseLinear(48, 40, sparsity=0.8), torch.nn.ReLU(),
                                sl.SparseLinear(40, 10, sparsity=0.7))
    algo = sl.SET(sparsity=0.8, drop_fraction=0.3, update_freq=3, seed=7)
    model.apply(algo)
    opt = torch.optim.AdamW(model.parameters(), lr=1e-2)
    return model, algo, opt


def _step(model, algo, opt, i):
    g = torch.Generator().manual_seed(100 + i)
    x = torch.randn(32, 48, generator=g).to(dev())
    y = torch.randint(0, 10, (32,), generator=g).to(dev())
    opt.zero_grad(set_to_none=True)
    loss = torch.nn.functional.cross_entropy(model(x), y)
    loss.backward()
    opt.step()
    algo.step()
    return float(loss.item())


def _masks(model):
    from sparsecore_b200 import SparseLinear

    return [(m._csr.col_indices.cpu().numpy().copy(), m._csr.values.detach().cpu().numpy().copy(),
             m._csr.topology_version) for m in model.modules() if isinstance(m, SparseLinear)]


@pytest.mark.parametrize("resume_seed", [0, 123])
def test_resume_continues_bit_identically(tmp_path, resume_seed):
    from sparsecore_b200 import checkpoint

    model, algo, opt = _make(0)
    for i in range(5):
        _step(model, algo, opt, i)  # one SET update at step 3
    path = tmp_path / "ck.pt"
    checkpoint.save(path, model, opt, algo, extra={"step": 5})
    ref = [_step(model, algo, opt, i) for i in range(5, 11)]  # updates at 6 and 9
    ref_masks = _masks(model)

    model2, algo2, opt2 = _make(resume_seed)
    assert checkpoint.load(path, model2, opt2, algo2) == {"step": 5}
    got = [_step(model2, algo2, opt2, i) for i in range(5, 11)]
    assert got == ref
    for (c1, v1, t1), (c2, v2, t2) in zip(ref_masks, _masks(model2)):
        assert np.array_equal(c1, c2) and np.array_equal(v1.view(np.int32), v2.view(np.int32))
        assert t1 == t2
    for m in model2.modules():
        if hasattr(m, "_csr"):
            m._csr.assert_invariants()
            assert m._values.data_ptr() == m._csr.values.data_ptr()
