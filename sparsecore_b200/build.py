"""Build the sparsecore_b200 CUDA library in-tree.

    python -m sparsecore_b200.build            # -> sparsecore_b200/_lib/libsparsecore_b200.so

One shared library with a plain C ABI (include/sparsecore_b200.h), compiled
for sm_100a only.  No fast-math: the kernels' bit-exactness depends on IEEE
fp32 semantics (explicit fmaf / __fadd_rn, denormals preserved).
"""
from __future__ import annotations

import glob
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
LIB_DIR = os.path.join(HERE, "_lib")
LIB_NAME = "libsparsecore_b200.so"
LIB_PATH = os.path.join(LIB_DIR, LIB_NAME)

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo", "-O3", "-std=c++17",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
]
LINK_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-cudart", "shared"]


def nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found: the sparsecore_b200 CUDA library cannot be built")
    return cand


def sources() -> list[str]:
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def _stale() -> bool:
    if not os.path.exists(LIB_PATH):
        return True
    t = os.path.getmtime(LIB_PATH)
    deps = sources() + glob.glob(os.path.join(CSRC, "*.cuh"))
    deps.append(os.path.join(HERE, "..", "include", "sparsecore_b200.h"))
    return any(os.path.getmtime(d) > t for d in deps if os.path.exists(d))


def build(force: bool = False, verbose: bool = False) -> str:
    """Compile every csrc/*.cu to an object (in parallel), then link the
    shared library."""
    if not force and not _stale():
        return LIB_PATH
    from concurrent.futures import ThreadPoolExecutor

    os.makedirs(LIB_DIR, exist_ok=True)
    obj_dir = os.path.join(LIB_DIR, "obj")
    os.makedirs(obj_dir, exist_ok=True)
    cc = nvcc()

    def compile_one(src):
        obj = os.path.join(obj_dir, os.path.basename(src) + ".o")
        cmd = [cc, *NVCC_FLAGS, "-Xptxas", "-v", "-c", src, "-o", obj]
        res = subprocess.run(cmd, capture_output=True, text=True)
        return obj, cmd, res

    with ThreadPoolExecutor(max_workers=max(1, min(len(sources()), os.cpu_count() or 1))) as ex:
        results = list(ex.map(compile_one, sources()))
    log = []
    failed = False
    for _, cmd, res in results:
        log.append(" ".join(cmd) + "\n" + res.stdout + res.stderr)
        failed |= res.returncode != 0
    tmp = LIB_PATH + ".tmp"
    if not failed:
        cmd = [cc, *LINK_FLAGS, *[o for o, _, _ in results], "-o", tmp]
        res = subprocess.run(cmd, capture_output=True, text=True)
        log.append(" ".join(cmd) + "\n" + res.stdout + res.stderr)
        failed = res.returncode != 0
    with open(os.path.join(LIB_DIR, "build.log"), "w") as f:
        f.write("\n".join(log))
    if verbose:
        print("\n".join(log))
    if failed:
        sys.stderr.write("\n".join(log))
        raise RuntimeError("nvcc failed building sparsecore_b200 (see _lib/build.log)")
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
