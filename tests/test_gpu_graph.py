"""CUDA-graph replay of a training step matches eager execution bit for bit,
across a SET update that forces a re-capture."""
import pytest
import torch

from gpu_helpers import dev

pytestmark = pytest.mark.gpu


def _setup():
    import sparsecore_b200 as sl

    torch.manual_seed(0)
    model = torch.nn.Sequential(sl.SparseLinear(64, 48, sparsity=0.8), torch.nn.ReLU(),
                                sl.SparseLinear(48, 10, sparsity=0.7))
    algo = sl.SET(sparsity=0.8, drop_fraction=0.3, update_freq=4, seed=1)
    model.apply(algo)
    opt = torch.optim.SGD(model.parameters(), lr=0.05)
    g = torch.Generator().manual_seed(9)
    x = torch.randn(40, 64, generator=g).to(dev())
    y = torch.randint(0, 10, (40,), generator=g).to(dev())

    def train(xb, yb):
        opt.zero_grad(set_to_none=True)
        loss = torch.nn.functional.cross_entropy(model(xb), yb)
        loss.backward()
        opt.step()
        return loss

    return model, algo, train, x, y


def test_graph_replay_matches_eager_across_topology_updates():
    from sparsecore_b200.graph import GraphedStep

    model, algo, train, x, y = _setup()
    eager = []
    for _ in range(10):
        eager.append(float(train(x, y).item()))
        algo.step()

    model2, algo2, train2, x2, y2 = _setup()
    train2(x2, y2)  # eager warm-up step (lazy initialisation), as the graph requires
    algo2.step()
    gs = GraphedStep(model2, train2, (x2, y2))
    graphed = [eager[0]]
    for _ in range(9):
        graphed.append(float(gs().item()))
        algo2.step()
    assert graphed == eager
    assert gs.captures == 3  # initial + after the updates at steps 4 and 8
