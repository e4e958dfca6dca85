"""Build ``libb2d.so`` (the C ABI in include/b2d.h) in-tree with nvcc.

The library is compiled for sm_100a only.  ``build()`` is idempotent: it
rebuilds when a source under ``csrc/`` or ``include/`` is newer than the
library.  The built file sits next to this module so it travels with the
repository snapshot to the GPU host.
"""

from __future__ import annotations

import glob
import os
import shutil
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libb2d.so")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC,-O3,-fvisibility=hidden",
    "-shared", "--expt-relaxed-constexpr",
    "-Xptxas", "-v",
]


def sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def _deps():
    return sources() + glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(REPO, "include", "*.h"))


def needs_build() -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    return any(os.path.getmtime(p) > t for p in _deps())


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def build(force: bool = False, verbose: bool = False) -> str:
    """Compile csrc/*.cu into libb2d.so (sm_100a).  Returns the library path."""
    if not force and not needs_build():
        return LIB
    tmp = LIB + ".tmp"
    cmd = [nvcc(), *NVCC_FLAGS, "-o", tmp, *sources(), "-lcudart"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    log = r.stdout + r.stderr
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed ({r.returncode}):\n{log}")
    with open(os.path.join(HERE, "libb2d.build.log"), "w") as f:
        f.write(" ".join(cmd) + "\n" + log)
    if verbose:
        print(log)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    build(force=True, verbose=True)
