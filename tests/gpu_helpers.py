"""Shared helpers for the GPU parity tests."""
import hashlib

import numpy as np
import torch


def dev():
    return torch.device("cuda", 0)


def csr_from_golden(golden, prefix):
    import sparsecore_b200 as sl

    a = golden.arrays
    M, K = (int(v) for v in a[prefix + "shape"])
    return sl.PaddedCSR(M, K, a[prefix + "values"], a[prefix + "cols"], a[prefix + "row_start"],
                        a[prefix + "row_nnz"], a[prefix + "row_capacity"], device=dev())


def bits(t):
    a = t.detach().float().contiguous().cpu().numpy() if isinstance(t, torch.Tensor) else np.asarray(t, np.float32)
    return np.ascontiguousarray(a, np.float32).view(np.int32)


def bits_equal(a, b):
    x, y = bits(a), bits(b)
    return x.shape == y.shape and np.array_equal(x, y)


def host(t):
    return t.detach().cpu().numpy() if isinstance(t, torch.Tensor) else np.asarray(t)


def csr_matches(W, golden, prefix):
    a = golden.arrays
    return (bits_equal(W.values, a[prefix + "values"])
            and np.array_equal(host(W.col_indices), a[prefix + "cols"])
            and np.array_equal(host(W.row_start), a[prefix + "row_start"])
            and np.array_equal(host(W.row_nnz), a[prefix + "row_nnz"])
            and np.array_equal(host(W.row_capacity), a[prefix + "row_capacity"]))


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def oracle_csr(W):
    from oracle import oracle as O

    return O.CSR(W.nrows, W.ncols, host(W.values).copy(), host(W.col_indices).copy(),
                 host(W.row_start).copy(), host(W.row_nnz).copy(), host(W.row_capacity).copy())


def launched_kernels(fn):
    """Run ``fn`` and return (its result, [the kernel its last SpMM / SDDMM
    dispatch launched]) as the library records it (sl_last_kernel), so a
    parity test can assert which kernel produced the values it checks."""
    from sparsecore_b200 import _native as N

    out = fn()
    torch.cuda.synchronize()
    return out, [N.lib().sl_last_kernel().decode()]


def random_csr(M, K, density, seed, block=None, device=None):
    """PaddedCSR from a seeded uniform mask (values N(0,1)); ``block`` =
    (rows, cols) of a fully dense top-left block."""
    import sparsecore_b200 as sl

    g = torch.Generator().manual_seed(seed)
    mask = torch.rand(M, K, generator=g) < density
    if block is not None:
        mask[:block[0], :block[1]] = True
    Wd = torch.randn(M, K, generator=g) * mask
    return sl.PaddedCSR.from_dense(Wd.to(device or dev()))
