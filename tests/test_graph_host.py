"""GraphedStep's capture bookkeeping on the CPU, with fakes for the CUDA
graph: one graph per variant key, every variant dropped and re-captured when
any layer's topology_version changes, replays otherwise."""
import types

import pytest
import torch


class _FakeGraph:
    replays = 0

    def replay(self):
        _FakeGraph.replays += 1


class _FakeCtx:
    def __init__(self, g):
        pass

    def __enter__(self):
        return self

    def __exit__(self, *a):
        return False


@pytest.fixture
def graphed(monkeypatch):
    from sparsecore_b200 import graph, ops
    from sparsecore_b200.nn import SparseLinear

    monkeypatch.setattr(torch.cuda, "CUDAGraph", _FakeGraph)
    monkeypatch.setattr(torch.cuda, "graph", _FakeCtx)
    monkeypatch.setattr(torch.cuda, "synchronize", lambda *a, **k: None)
    monkeypatch.setattr(ops, "_cached_transpose", lambda csr: None)
    status_checks = []
    monkeypatch.setattr(graph.N, "check_device_status", lambda dev: status_checks.append(dev))
    layers = []
    for _ in range(2):
        m = SparseLinear.__new__(SparseLinear)
        torch.nn.Module.__init__(m)
        m._csr = types.SimpleNamespace(topology_version=0, values=torch.zeros(1))
        layers.append(m)
    model = torch.nn.Sequential(*layers)
    monkeypatch.setattr(graph, "status_checks", status_checks, raising=False)
    return graph, model, layers


def test_one_graph_per_variant_and_recapture_on_topology_change(graphed):
    graph, model, layers = graphed
    calls = []
    state = {"variant": (False, 0)}

    def step():
        calls.append(state["variant"])
        return torch.tensor(float(len(calls)))

    gs = graph.GraphedStep(model, step, (), variant=lambda: state["variant"])
    _FakeGraph.replays = 0
    for _ in range(3):
        gs()
    assert gs.captures == 1 and _FakeGraph.replays == 3
    assert len(graph.status_checks) == 1  # the device status is read at each capture
    state["variant"] = (True, 0)   # e.g. RigL about to clone X / dY
    gs()
    gs()
    assert gs.captures == 2
    state["variant"] = (False, 0)  # back to the clone-free graph: no re-capture
    gs()
    assert gs.captures == 2 and _FakeGraph.replays == 6
    layers[1]._csr.topology_version += 3  # a router update rewrote rows
    gs()
    assert gs.captures == 3
    state["variant"] = (True, 0)   # variants were dropped with the old topology
    gs()
    assert gs.captures == 4
    assert calls == [(False, 0), (True, 0), (False, 0), (True, 0)]


def test_no_variant_means_single_graph(graphed):
    graph, model, layers = graphed
    gs = graph.GraphedStep(model, lambda: torch.zeros(()), ())
    for _ in range(4):
        gs()
    assert gs.captures == 1
    layers[0]._csr.topology_version += 1
    gs()
    assert gs.captures == 2


def test_rigl_graph_variant_keys():
    """RigL capture gating (host only, no layers attached): capture="update_step"
    clones only before an update step, and the key's generation moves on
    after every update so no cloning graph outlives its clone buffers."""
    import sparsecore_b200 as sl

    every = sl.RigL(sparsity=0.9, update_freq=3, capture="every_step")
    upd = sl.RigL(sparsity=0.9, update_freq=3, capture="update_step")
    seen_every, seen_upd = [], []
    for _ in range(7):
        seen_every.append(every.graph_variant())
        seen_upd.append(upd.graph_variant())
        every.step()
        upd.step()
    assert seen_every == [(True, 0)] * 3 + [(True, 1)] * 3 + [(True, 2)]
    assert seen_upd == [(False, 0), (False, 0), (True, 0), (False, 0), (False, 0), (True, 1), (False, 0)]
    with pytest.raises(ValueError):
        sl.RigL(sparsity=0.9, capture="sometimes")
