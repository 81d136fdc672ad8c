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


def _setup_rigl(capture):
    import sparsecore_b200 as sl

    torch.manual_seed(0)
    model = torch.nn.Sequential(sl.SparseLinear(64, 48, sparsity=0.8), torch.nn.ReLU(),
                                sl.SparseLinear(48, 10, sparsity=0.7))
    algo = sl.RigL(sparsity=0.8, drop_fraction=0.3, update_freq=3, seed=1, capture=capture)
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


@pytest.mark.parametrize("capture", ["every_step", "update_step"])
def test_graph_variants_for_rigl_capture(capture):
    """RigL clones X / dY inside the graph: with capture="update_step" the
    step keeps a graph with the clones and one without (keyed by
    graph_variant), and replay matches eager every-step capture exactly."""
    from sparsecore_b200.graph import GraphedStep

    model, algo, train, x, y = _setup_rigl("every_step")
    eager = []
    for _ in range(10):
        eager.append(float(train(x, y).item()))
        algo.step()
    ref_cols = [m._csr.col_indices.cpu() for m in model if hasattr(m, "_csr")]

    model2, algo2, train2, x2, y2 = _setup_rigl(capture)
    train2(x2, y2)
    algo2.step()
    gs = GraphedStep(model2, train2, (x2, y2), variant=algo2.graph_variant)
    graphed = [eager[0]]
    for _ in range(9):
        graphed.append(float(gs().item()))
        algo2.step()
    assert graphed == eager
    cols = [m._csr.col_indices.cpu() for m in model2 if hasattr(m, "_csr")]
    assert all(torch.equal(a, b) for a, b in zip(ref_cols, cols))
    assert model2[0]._csr.topology_version > 0
    # Updates follow steps 2, 5 and 8.  every_step: one graph per topology /
    # clone generation (captured at steps 1, 3, 6, 9); update_step: a
    # clone-free graph per topology (1, 3, 6, 9) plus the cloning one before
    # each update (2, 5, 8).
    assert gs.captures == (4 if capture == "every_step" else 7)


class _FusedFFN(torch.nn.Module):
    """Biased FFN pair through sparse_mlp (bias and GELU in the first
    layer's forward kernel, the second bias in the output transpose)."""

    def __init__(self):
        import sparsecore_b200 as sl

        super().__init__()
        self.fc1 = sl.SparseLinear(64, 96, sparsity=0.8)
        self.fc2 = sl.SparseLinear(96, 10, sparsity=0.7)

    def forward(self, x):
        import sparsecore_b200 as sl

        return sl.sparse_mlp(x, self.fc1, self.fc2, "gelu")


def test_graph_replay_of_fused_biased_ffn_matches_eager():
    import sparsecore_b200 as sl
    from sparsecore_b200.graph import GraphedStep

    def setup():
        torch.manual_seed(0)
        model = _FusedFFN()
        algo = sl.SET(sparsity=0.8, drop_fraction=0.3, update_freq=4, seed=1)
        opt = torch.optim.SGD(model.parameters(), lr=0.05)
        g = torch.Generator().manual_seed(9)
        x = torch.randn(300, 64, generator=g).to(dev())
        y = torch.randint(0, 10, (300,), generator=g).to(dev())
        model.apply(algo)

        def train(xb, yb):
            opt.zero_grad(set_to_none=True)
            loss = torch.nn.functional.cross_entropy(model(xb), yb)
            loss.backward()
            opt.step()
            return loss

        return algo, train, x, y, model

    algo, train, x, y, model = setup()
    eager = []
    for _ in range(9):
        eager.append(float(train(x, y).item()))
        algo.step()
    algo2, train2, x2, y2, model2 = setup()
    train2(x2, y2)
    algo2.step()
    gs = GraphedStep(model2, train2, (x2, y2))
    graphed = [eager[0]]
    for _ in range(8):
        graphed.append(float(gs().item()))
        algo2.step()
    assert graphed == eager
    assert torch.equal(model.fc1.bias, model2.fc1.bias) and torch.equal(model.fc2.bias, model2.fc2.bias)
