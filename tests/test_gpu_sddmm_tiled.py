"""Tiled SDDMM (the weight-gradient kernel of every transformer-sized
training step: N >= 1024, N % 32 == 0, live density 2-40%) against the C
oracle's restatement of the reference AVX2 kernel
(csrc/kernels/spmm_grad_avx2.cpp:73-259), bit for bit.  Every case first
asserts, from the profiler's kernel list, that the tiled kernel is the one
that ran, so the comparison cannot silently fall back to the per-slot
kernels."""
import pytest
import torch

from gpu_helpers import bits_equal, dev, launched_kernels, oracle_csr, random_csr

pytestmark = pytest.mark.gpu

TILED = "sddmm_tiled_kernel"


def _dw_checked(W, dY, X, expect_tiled=True):
    from sparsecore_b200 import ops

    dw, names = launched_kernels(lambda: ops._sddmm_raw(W, dY, X))
    ran_tiled = any(TILED in n for n in names)
    assert ran_tiled == expect_tiled, names
    return dw


def _case(M, K, density, N, seed, block=None):
    W = random_csr(M, K, density, seed, block=block)
    g = torch.Generator().manual_seed(seed + 1)
    X = torch.randn(K, N, generator=g)
    dY = torch.randn(M, N, generator=g)
    return W, X, dY


# Transformer layer shapes (W is out x in): config 5 ffn_up / ffn_down at 90%,
# qkv / o at 70%; config 4 ffn_up and qkv; the config-3 4096^2 at 90%.
LAYERS = [
    ("cfg5_ffn_up", 3072, 768, 0.10, 2048),
    ("cfg5_ffn_down", 768, 3072, 0.10, 2048),
    ("cfg5_qkv", 2304, 768, 0.30, 1024),
    ("cfg5_o", 768, 768, 0.30, 2048),
    ("cfg4_ffn_up", 1536, 384, 0.10, 2048),
    ("cfg4_qkv", 1152, 384, 0.30, 1024),
    ("cfg3_4096sq_90", 4096, 4096, 0.10, 2048),
]


@pytest.mark.parametrize("name,M,K,density,N", LAYERS, ids=[c[0] for c in LAYERS])
def test_tiled_sddmm_layer_shapes_vs_oracle(name, M, K, density, N):
    from oracle import oracle as O

    W, X, dY = _case(M, K, density, N, seed=M * 3 + K)
    dw = _dw_checked(W, dY.to(dev()), X.to(dev()))
    assert bits_equal(dw, O.sddmm(oracle_csr(W), dY.numpy(), X.numpy())), name


def test_tiled_sddmm_config5_ffn_up_at_training_width():
    """The headline step's dominant launch: ffn_up at N = 16384 (32 x 512
    tokens), and the X-stationary forward the same layer takes by default."""
    from oracle import oracle as O

    import sparsecore_b200 as sl

    W, X, dY = _case(3072, 768, 0.10, 16384, seed=5)
    Wo = oracle_csr(W)
    dw = _dw_checked(W, dY.to(dev()), X.to(dev()))
    assert bits_equal(dw, O.sddmm(Wo, dY.numpy(), X.numpy()))
    y, names = launched_kernels(lambda: sl.spmm(W, X.to(dev())))
    assert any("spmm_xs_kernel" in n for n in names), names
    assert bits_equal(y, O.spmm(Wo, X.numpy()))


@pytest.mark.parametrize("seg", ["1", "0", "auto"])
@pytest.mark.parametrize("tc", ["64", "128", "256"])
@pytest.mark.parametrize("order", ["row", "col"])
def test_tiled_sddmm_tile_widths_and_orders(tc, order, seg, monkeypatch):
    """Every tile width and both tile orders, with slot (default) and
    segmented batches and the per-shape timed choice, on ragged edges (M, K not multiples of any tile) with a
    dense block that puts thousands of slots in one tile (several batches
    per tile)."""
    from oracle import oracle as O

    W, X, dY = _case(1000, 1100, 0.06, 1024, seed=17, block=(130, 300))
    ref = O.sddmm(oracle_csr(W), dY.numpy(), X.numpy())
    monkeypatch.setenv("SPARSECORE_B200_DW_SEG", seg)
    monkeypatch.setenv("SPARSECORE_B200_DW_TC", tc)
    monkeypatch.setenv("SPARSECORE_B200_DW_ORDER", order)
    assert bits_equal(_dw_checked(W, dY.to(dev()), X.to(dev())), ref)


@pytest.mark.parametrize("density", [0.021, 0.39])
def test_tiled_sddmm_density_limits(density):
    """Densities just inside the tiled kernel's 2-40% window."""
    from oracle import oracle as O

    W, X, dY = _case(700, 900, density, 1024, seed=int(density * 1000))
    dw = _dw_checked(W, dY.to(dev()), X.to(dev()))
    assert bits_equal(dw, O.sddmm(oracle_csr(W), dY.numpy(), X.numpy()))


def test_outside_window_takes_the_per_slot_kernel():
    """Outside the window (here 60% live) the per-slot kernel runs, and
    agrees with the oracle too."""
    from oracle import oracle as O

    W, X, dY = _case(300, 200, 0.6, 1024, seed=3)
    dw = _dw_checked(W, dY.to(dev()), X.to(dev()), expect_tiled=False)
    assert bits_equal(dw, O.sddmm(oracle_csr(W), dY.numpy(), X.numpy()))
