"""GPU: SET / RigL rewrites vs the reference's golden topologies (bit-exact),
SparseLinear init/forward/backward, and the config-2 MLP + SET trajectory."""
import types

import numpy as np
import pytest
import torch

from gpu_helpers import bits_equal, csr_from_golden, csr_matches, dev, host, sha

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("idx", range(7))
def test_set_matches_reference(golden, idx):
    import sparsecore_b200 as sl

    fin, fout, s, df, seed, tie, nup = golden.meta["set_cases"][idx]
    p = f"set{idx}_"
    algo = sl.SET(sparsity=s, drop_fraction=df, update_freq=1, seed=seed)
    versions = golden[p + "versions"]
    W = csr_from_golden(golden, p + "in_")
    prev_v = 0
    for u in range(nup):
        layer = types.SimpleNamespace(_csr=W)
        v0 = W.topology_version
        algo._update_layer(layer, algo._rng)
        assert csr_matches(W, golden, f"{p}out{u}_"), f"update {u}"
        W.assert_invariants()
        assert W.topology_version - v0 == int(versions[u]) - prev_v
        prev_v = int(versions[u])
        W = csr_from_golden(golden, f"{p}pert{u}_")


@pytest.mark.parametrize("idx", range(5))
def test_rigl_matches_reference(golden, idx):
    import sparsecore_b200 as sl

    fin, fout, s, df, kind = golden.meta["rigl_cases"][idx]
    p = f"rigl{idx}_"
    W = csr_from_golden(golden, p + "in_")
    algo = sl.RigL(sparsity=s, drop_fraction=df, update_freq=1, seed=0)
    layer = types.SimpleNamespace(_csr=W, in_features=fin, out_features=fout)
    G = torch.from_numpy(golden[p + "G"]).to(dev())
    algo._update_layer(layer, algo._rng, G=G)
    assert csr_matches(W, golden, p + "out_")
    assert W.topology_version == int(golden[p + "version"][0])
    W.assert_invariants()


def test_rigl_end_to_end_captures_and_grows():
    import sparsecore_b200 as sl

    torch.manual_seed(0)
    layer = sl.SparseLinear(64, 32, sparsity=0.9)
    algo = sl.RigL(sparsity=0.9, drop_fraction=0.3, update_freq=2, seed=0)
    layer.apply(algo)
    nnz0 = layer.nnz
    x = torch.randn(16, 64, device=dev())
    for _ in range(2):
        layer(x).pow(2).sum().backward()
        algo.step()
    assert layer._csr.topology_version > 0
    assert layer.nnz == nnz0
    layer._csr.assert_invariants()


def test_rigl_update_step_capture_matches_every_step():
    """capture="update_step" clones X / dY only before an update, and the
    rewritten topology is the same as with the reference's every-step
    capture."""
    import sparsecore_b200 as sl

    out = {}
    for mode in ("every_step", "update_step"):
        torch.manual_seed(0)
        layer = sl.SparseLinear(96, 48, sparsity=0.85)
        opt = torch.optim.SGD(layer.parameters(), lr=0.1)
        algo = sl.RigL(sparsity=0.85, drop_fraction=0.3, update_freq=3, seed=4, capture=mode)
        layer.apply(algo)
        xs = torch.randn(7, 20, 96, device=dev()).unbind(0)
        n_cap = []
        for x in xs:
            opt.zero_grad()
            layer(x).pow(2).sum().backward()
            n_cap.append(len(algo._captured))
            opt.step()
            algo.step()
        out[mode] = (host(layer._csr.col_indices), host(layer._csr.row_nnz),
                     host(layer._csr.values), layer._csr.topology_version, n_cap)
    a, b = out["every_step"], out["update_step"]
    assert a[3] == b[3] > 0
    assert np.array_equal(a[0], b[0]) and np.array_equal(a[1], b[1])
    assert bits_equal(a[2], b[2])
    assert a[4] == [1] * 7 and b[4] == [0, 0, 1, 0, 0, 1, 0]


def test_sparse_linear_init_matches_reference_draws():
    import sparsecore_b200 as sl

    torch.manual_seed(123)
    layer = sl.SparseLinear(50, 20, sparsity=0.8)
    torch.manual_seed(123)
    bound = 1.0 / np.sqrt(max(1.0, 50 * 0.2))
    Wd = torch.empty(20, 50)
    torch.nn.init.uniform_(Wd, -bound, bound)
    mask = torch.rand(20, 50) >= 0.8
    b = torch.empty(20)
    torch.nn.init.uniform_(b, -bound, bound)
    assert torch.equal(layer._csr.to_dense().cpu(), Wd * mask.float())
    assert torch.equal(layer.bias.detach().cpu(), b)
    assert layer._values.data_ptr() == layer._csr.values.data_ptr()
    assert "nnz=" in layer.extra_repr()
    assert abs(layer.density - layer.nnz / 1000) < 1e-12


def test_sparse_linear_matches_dense_torch():
    import sparsecore_b200 as sl

    torch.manual_seed(1)
    layer = sl.SparseLinear(96, 40, sparsity=0.7)
    x = torch.randn(3, 5, 96, device=dev(), requires_grad=True)
    y = layer(x)
    assert y.shape == (3, 5, 40)
    Wd = layer._csr.to_dense().detach().requires_grad_(True)
    xd = x.detach().clone().requires_grad_(True)
    yd = xd @ Wd.t() + layer.bias
    assert torch.allclose(y, yd, rtol=1e-5, atol=1e-5)
    gy = torch.randn_like(y)
    y.backward(gy)
    yd.backward(gy)
    assert torch.allclose(x.grad, xd.grad, rtol=1e-5, atol=1e-5)
    # live-slot gradient equals the dense gradient at the live positions
    W = layer._csr
    rs, rn, cols = host(W.row_start), host(W.row_nnz), host(W.col_indices)
    g = host(layer._values.grad)
    gd = host(Wd.grad)
    for i in range(W.nrows):
        for k in range(rn[i]):
            assert abs(g[rs[i] + k] - gd[i, cols[rs[i] + k]]) <= 1e-4 * (1 + abs(gd[i, cols[rs[i] + k]]))
    # padding slots get zero gradient
    pad = np.ones(W.total_capacity, bool)
    for i in range(W.nrows):
        pad[rs[i]:rs[i] + rn[i]] = False
    assert np.all(g[pad] == 0)


def test_state_dict_roundtrip_keeps_alias():
    import sparsecore_b200 as sl

    torch.manual_seed(5)
    a = sl.SparseLinear(30, 10, sparsity=0.5)
    torch.manual_seed(5)
    b = sl.SparseLinear(30, 10, sparsity=0.5)
    with torch.no_grad():
        a._values.mul_(3.0)
    b.load_state_dict(a.state_dict())
    assert torch.equal(b._csr.values, a._csr.values)
    assert b._values.data_ptr() == b._csr.values.data_ptr()


def test_mlp_set_trajectory_matches_reference(golden):
    """Config-2 MLP with SET, 250 steps, same seeds as the reference run on
    CPU.  SpMM/dW/dX are bit-exact; cross-entropy, bias add and SGD run in
    torch on the GPU, so the loss may drift in the last bits: tolerance."""
    import torch.nn as tnn
    import torch.nn.functional as F
    import sparsecore_b200 as sl

    m = golden.meta["mlp"]
    torch.manual_seed(0)
    model = tnn.Sequential(sl.SparseLinear(784, 512, sparsity=0.9), tnn.ReLU(),
                           sl.SparseLinear(512, 10, sparsity=0.9))
    g = torch.Generator().manual_seed(7)
    x = torch.randn(256, 784, generator=g).to(dev())
    y = torch.randint(0, 10, (256,), generator=g).to(dev())
    opt = torch.optim.SGD(model.parameters(), lr=0.1)
    algo = sl.SET(sparsity=0.9, drop_fraction=0.3, update_freq=100, seed=0)
    model.apply(algo)
    losses = []
    for _ in range(m["steps"]):
        opt.zero_grad()
        loss = F.cross_entropy(model(x), y)
        loss.backward()
        opt.step()
        algo.step()
        losses.append(float(loss.item()))
    ref = np.array(m["losses"])
    got = np.array(losses)
    assert np.max(np.abs(got - ref)) < 2e-4, np.max(np.abs(got - ref))
    assert [model[0]._csr.topology_version, model[2]._csr.topology_version] == m["versions"]
    same1 = sha(host(model[0]._csr.col_indices)) == m["sha_cols_fc1"]
    same2 = sha(host(model[2]._csr.col_indices)) == m["sha_cols_fc2"]
    print("mlp max|dloss|", float(np.max(np.abs(got - ref))), "topology identical:", same1, same2)


@pytest.mark.parametrize("idx", range(5))
def test_rigl_fused_grow_matches_reference(golden, idx):
    """The fused grow path (gradient GEMM with per-tile candidates, merge,
    no M x K buffer) on the reference's golden RigL cases: captured operands
    X = I, dY = G^T make the in-order dense gradient equal G exactly, so the
    topology must equal the reference's (ties and zero gradients included:
    those rows go to the host argpartition)."""
    import sparsecore_b200 as sl

    fin, fout, s, df, kind = golden.meta["rigl_cases"][idx]
    p = f"rigl{idx}_"
    W = csr_from_golden(golden, p + "in_")
    algo = sl.RigL(sparsity=s, drop_fraction=df, update_freq=1, seed=0)
    assert algo.fused_grow
    layer = types.SimpleNamespace(_csr=W, in_features=fin, out_features=fout)
    G = torch.from_numpy(golden[p + "G"])
    algo._captured[id(layer)] = {"X": torch.eye(fin).to(dev()), "dY": G.t().contiguous().to(dev())}
    algo._update_layer(layer, algo._rng)
    assert csr_matches(W, golden, p + "out_")
    assert W.topology_version == int(golden[p + "version"][0])
    W.assert_invariants()


@pytest.mark.parametrize("tiling", ["64", "128"])
@pytest.mark.parametrize("M,K,s,zero_rows", [(300, 700, 0.9, False), (1536, 384, 0.9, True),
                                             (200, 1100, 0.5, False)])
def test_rigl_fused_grow_equals_materialised_path(M, K, s, zero_rows, tiling, monkeypatch):
    """Fused and materialised grow paths on random layers (64- and 128-column
    GEMM tiles, ragged edges, long rows beyond the per-tile candidate cap),
    with rows of all-zero gradient (every candidate ties: host path) mixed
    in."""
    import sparsecore_b200 as sl

    monkeypatch.setenv("SPARSECORE_B200_DG", tiling)

    out = []
    for fused in (True, False):
        g = torch.Generator().manual_seed(M + K)
        mask = torch.rand(M, K, generator=g) >= s
        W = sl.PaddedCSR.from_dense((torch.randn(M, K, generator=g) * mask).to(dev()))
        X = torch.randn(64, K, generator=g)
        dY = torch.randn(64, M, generator=g)
        if zero_rows:
            dY[:, ::7] = 0.0
        algo = sl.RigL(sparsity=s, drop_fraction=0.3, update_freq=1, seed=0, fused_grow=fused)
        layer = types.SimpleNamespace(_csr=W, in_features=K, out_features=M)
        algo._captured[id(layer)] = {"X": X.to(dev()), "dY": dY.to(dev())}
        algo._update_layer(layer, algo._rng)
        W.assert_invariants()
        out.append((host(W.col_indices), host(W.row_nnz), host(W.values), W.topology_version))
    (a, b) = out
    assert np.array_equal(a[0], b[0]) and np.array_equal(a[1], b[1])
    assert bits_equal(a[2], b[2]) and a[3] == b[3]
