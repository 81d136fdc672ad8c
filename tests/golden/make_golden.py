"""Generate the golden fixtures in tests/golden/ from the REFERENCE itself.

Run here (where the reference sources are mounted), never on the GPU box:

    make -C oracle ref                       # builds oracle/_ref/refcore/_core*.so
    python tests/golden/make_golden.py [--ref <reference source tree>]

The reference's Python package is imported from its own source tree, with
its compiled `_core` taken from oracle/_ref/refcore (built from the
reference's own C++ sources by oracle/Makefile).  Every output stored here
is what the reference computes; inputs are seeded and stored alongside.
"""
from __future__ import annotations

import argparse
import hashlib
import importlib.util
import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))


def load_reference(ref_root: str):
    core_dir = os.path.join(REPO, "oracle", "_ref", "refcore")
    if not os.path.isdir(core_dir):
        raise SystemExit("build the reference core first: make -C oracle ref")
    pkg = os.path.join(ref_root, "sparselab")
    spec = importlib.util.spec_from_file_location(
        "sparselab", os.path.join(pkg, "__init__.py"),
        submodule_search_locations=[pkg, core_dir])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["sparselab"] = mod
    spec.loader.exec_module(mod)
    return mod, sys.modules["sparselab._core"]


def csr_arrays(W) -> dict:
    return {
        "shape": np.array([W.nrows, W.ncols], np.int64),
        "values": np.array(W.values, np.float32),
        "cols": np.array(W.col_indices, np.int32),
        "row_start": np.array(W.row_start, np.int32),
        "row_nnz": np.array(W.row_nnz, np.int32),
        "row_capacity": np.array(W.row_capacity, np.int32),
    }


def prefixed(prefix: str, d: dict) -> dict:
    return {f"{prefix}{k}": v for k, v in d.items()}


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


# Kernel cases: (M, K, N, sparsity, seed).  Cover N mod 16 residues, N=1,
# tiny/empty rows, dense rows, 99% sparsity.
KERNEL_CASES = [
    (64, 80, 33, 0.9, 1), (128, 128, 8, 0.8, 2), (100, 300, 1, 0.5, 3), (50, 70, 17, 0.0, 4),
    (33, 65, 130, 0.99, 5), (40, 40, 24, 0.3, 6), (17, 250, 255, 0.95, 7), (96, 64, 64, 0.9, 8),
    (7, 5, 3, 0.5, 9), (200, 64, 100, 0.7, 10), (64, 512, 96, 0.9, 11), (31, 47, 47, 0.6, 12),
]


def gen_kernel_cases(sl, core, out: dict, meta: dict) -> None:
    for idx, (M, K, N, s, seed) in enumerate(KERNEL_CASES):
        W = sl.PaddedCSR.random(M, K, sparsity=s, seed=seed)
        g = torch.Generator().manual_seed(1000 + seed)
        X = torch.randn(K, N, generator=g).numpy()
        dY = torch.randn(M, N, generator=g).numpy()
        Y = core.spmm_simd(W, X)
        dW = core.spmm_grad_w_simd(W, dY, X)
        WT, perm = sl.layout.transpose_with_perm(W)
        dX = core.spmm_simd(WT, dY)
        G = core.dense_grad(dY, X)
        p = f"k{idx}_"
        out.update(prefixed(p + "W_", csr_arrays(W)))
        out.update(prefixed(p + "WT_", csr_arrays(WT)))
        out[p + "perm"] = np.asarray(perm, np.int64)
        out[p + "X"], out[p + "dY"] = X, dY
        out[p + "Y"], out[p + "dW"], out[p + "dX"], out[p + "G"] = Y, dW, dX, G
    meta["kernel_cases"] = KERNEL_CASES


def gen_cfg1(sl, core, meta: dict) -> None:
    """Config 1 (SparseLinear 784->256, 90%): inputs from seeds, outputs as
    hashes (too large to store) plus a few values."""
    torch.manual_seed(0)
    layer = sl.SparseLinear(784, 256, sparsity=0.9, bias=False)
    W = layer._csr
    g = torch.Generator().manual_seed(1)
    X = torch.randn(784, 256, generator=g).numpy()
    dY = torch.randn(256, 256, generator=g).numpy()
    Y = core.spmm_simd(W, X)
    dW = core.spmm_grad_w_simd(W, dY, X)
    WT, perm = sl.layout.transpose_with_perm(W)
    dX = core.spmm_simd(WT, dY)
    meta["cfg1"] = {
        "recipe": "torch.manual_seed(0); SparseLinear(784,256,sparsity=0.9,bias=False); "
                  "g=torch.Generator().manual_seed(1); X=randn(784,256,g); dY=randn(256,256,g)",
        "nnz": int(W.nnz), "total_capacity": int(W.total_capacity),
        "sha_values": sha(np.array(W.values)), "sha_cols": sha(np.array(W.col_indices)),
        "sha_X": sha(X), "sha_dY": sha(dY),
        "sha_Y": sha(Y), "sha_dW": sha(dW), "sha_dX": sha(dX),
        "sha_WT_cols": sha(np.array(WT.col_indices)), "sha_perm": sha(np.asarray(perm, np.int64)),
        "Y_00": float(Y[0, 0]), "dW_sum": float(np.float64(dW).sum()),
    }


def randomize_values(W, rng: np.random.Generator, tie_frac: float = 0.0) -> None:
    """Give live slots varied magnitudes (and optionally exact ties)."""
    vals = np.asarray(W.values)
    rs, rn = np.asarray(W.row_start), np.asarray(W.row_nnz)
    for i in range(W.nrows):
        n = int(rn[i])
        v = rng.standard_normal(n).astype(np.float32)
        if tie_frac > 0:
            t = rng.random(n) < tie_frac
            v[t] = np.float32(0.25) * np.sign(v[t])
        vals[rs[i]:rs[i] + n] = v


SET_CASES = [  # (in, out, sparsity, drop_fraction, seed, tie_frac, n_updates)
    (64, 48, 0.9, 0.3, 0, 0.0, 3), (100, 40, 0.5, 0.3, 1, 0.0, 2), (30, 20, 0.95, 0.5, 2, 0.0, 2),
    (80, 64, 0.9, 0.3, 3, 0.3, 2), (16, 16, 0.2, 0.9, 4, 0.0, 2), (200, 100, 0.99, 0.3, 5, 0.0, 2),
    (784, 128, 0.9, 0.3, 6, 0.0, 1),
]


def gen_set_cases(sl, out: dict, meta: dict) -> None:
    for idx, (fin, fout, s, df, seed, tie, nup) in enumerate(SET_CASES):
        torch.manual_seed(100 + idx)
        layer = sl.SparseLinear(fin, fout, sparsity=s, bias=False)
        randomize_values(layer._csr, np.random.default_rng(200 + idx), tie)
        p = f"set{idx}_"
        out.update(prefixed(p + "in_", csr_arrays(layer._csr)))
        algo = sl.SET(sparsity=s, drop_fraction=df, update_freq=1, seed=seed)
        layer.apply(algo)
        versions = []
        for u in range(nup):
            algo.update()
            versions.append(int(layer._csr.topology_version))
            out.update(prefixed(f"{p}out{u}_", csr_arrays(layer._csr)))
            # perturb the surviving values between updates (deterministic)
            randomize_values(layer._csr, np.random.default_rng(300 + 10 * idx + u), tie)
            out.update(prefixed(f"{p}pert{u}_", csr_arrays(layer._csr)))
        out[p + "versions"] = np.array(versions, np.int64)
    meta["set_cases"] = SET_CASES


RIGL_CASES = [  # (in, out, sparsity, drop_fraction, g_kind)
    (64, 48, 0.9, 0.3, "normal"), (100, 40, 0.5, 0.3, "normal"), (40, 24, 0.8, 0.5, "ties"),
    (30, 30, 0.95, 0.9, "zeros"), (120, 64, 0.9, 0.3, "normal"),
]


def gen_rigl_cases(sl, core, out: dict, meta: dict) -> None:
    for idx, (fin, fout, s, df, kind) in enumerate(RIGL_CASES):
        torch.manual_seed(400 + idx)
        layer = sl.SparseLinear(fin, fout, sparsity=s, bias=False)
        randomize_values(layer._csr, np.random.default_rng(500 + idx))
        rng = np.random.default_rng(600 + idx)
        G = rng.standard_normal((fout, fin)).astype(np.float32)
        if kind == "ties":
            G = np.round(G * 2).astype(np.float32) / 2  # many exact ties
        elif kind == "zeros":
            G[rng.random(G.shape) < 0.7] = 0.0
        p = f"rigl{idx}_"
        out.update(prefixed(p + "in_", csr_arrays(layer._csr)))
        out[p + "G"] = G
        algo = sl.RigL(sparsity=s, drop_fraction=df, update_freq=1, seed=0)
        layer.apply(algo)
        algo._captured[id(layer)] = {"X": torch.zeros(1, fin), "dY": torch.zeros(1, fout)}
        saved = core.dense_grad
        core.dense_grad = lambda dY, X, _G=G: _G.copy()
        try:
            algo.update()
        finally:
            core.dense_grad = saved
        out.update(prefixed(p + "out_", csr_arrays(layer._csr)))
        out[p + "version"] = np.array([layer._csr.topology_version], np.int64)
    meta["rigl_cases"] = RIGL_CASES


def gen_mlp_trajectory(sl, meta: dict, steps: int = 250) -> None:
    """Config-2 MLP (784->512->10, both 90%, SET every 100 steps) trained by the
    reference on CPU: per-step losses and the topology hash after training."""
    import torch.nn as tnn
    import torch.nn.functional as F

    torch.manual_seed(0)
    model = tnn.Sequential(sl.SparseLinear(784, 512, sparsity=0.9), tnn.ReLU(),
                           sl.SparseLinear(512, 10, sparsity=0.9))
    g = torch.Generator().manual_seed(7)
    x = torch.randn(256, 784, generator=g)
    y = torch.randint(0, 10, (256,), generator=g)
    opt = torch.optim.SGD(model.parameters(), lr=0.1)
    algo = sl.SET(sparsity=0.9, drop_fraction=0.3, update_freq=100, seed=0)
    model.apply(algo)
    losses = []
    for _ in range(steps):
        opt.zero_grad()
        loss = F.cross_entropy(model(x), y)
        loss.backward()
        opt.step()
        algo.step()
        losses.append(float(loss.item()))
    meta["mlp"] = {
        "recipe": "torch.manual_seed(0); Sequential(SparseLinear(784,512,.9), ReLU, "
                  "SparseLinear(512,10,.9)); g=Generator().manual_seed(7); x=randn(256,784,g); "
                  "y=randint(0,10,(256,),g); SGD lr 0.1; SET(.9,.3,100,seed=0)",
        "steps": steps, "losses": losses,
        "sha_cols_fc1": sha(np.array(model[0]._csr.col_indices)),
        "sha_cols_fc2": sha(np.array(model[2]._csr.col_indices)),
        "versions": [int(model[0]._csr.topology_version), int(model[2]._csr.topology_version)],
    }


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("SPARSELAB_REF"),
                    help="root of the reference source tree (or set SPARSELAB_REF)")
    args = ap.parse_args()
    if not args.ref:
        ap.error("the reference source tree is required: --ref DIR or SPARSELAB_REF=DIR")
    sl, core = load_reference(args.ref)
    meta = {"numpy": np.__version__, "torch": torch.__version__, "reference": "sparselab 0.2.x"}
    arrays: dict = {}
    gen_kernel_cases(sl, core, arrays, meta)
    gen_cfg1(sl, core, meta)
    gen_set_cases(sl, arrays, meta)
    gen_rigl_cases(sl, core, arrays, meta)
    gen_mlp_trajectory(sl, meta)
    np.savez_compressed(os.path.join(HERE, "golden.npz"), **arrays)
    with open(os.path.join(HERE, "golden.json"), "w") as f:
        json.dump(meta, f, indent=1)
    print("wrote", len(arrays), "arrays")


if __name__ == "__main__":
    main()
