"""Build the sm_100a shared libraries in-tree with nvcc.

    python diffusion-llm_b200/build.py [--force]

lib/libbd3attn.so             the product: the C ABI of include/bd3_attn.h (csrc/capi.cu
                              and the kernel headers it includes, one translation unit)
tests/diag/libbd3diag.so      tests only: the tcgen05 operand layouts and the FMA-pipe
                              exponential checked in isolation (tests/diag/diag_umma.cu)

A library is rebuilt when any of its sources, a file under csrc/ or include/ is newer.
"""

from __future__ import annotations

import glob
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "lib")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-shared", "-Xcompiler", "-fPIC",
         "-Xcompiler", "-fvisibility=hidden", "--expt-relaxed-constexpr"]

DIAG = os.path.join(REPO, "tests", "diag")

# output path -> sources
TARGETS = {
    os.path.join(LIB, "libbd3attn.so"): [os.path.join(CSRC, "capi.cu")],
    os.path.join(DIAG, "libbd3diag.so"): [os.path.join(DIAG, "diag_umma.cu")],
}


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _deps_mtime(srcs: list[str]) -> float:
    files = glob.glob(os.path.join(CSRC, "*")) + glob.glob(os.path.join(REPO, "include", "*.h"))
    return max(os.path.getmtime(f) for f in files + srcs)


def _build_one(out: str, srcs: list[str], force: bool) -> str:
    name = os.path.relpath(out, REPO)
    if not force and os.path.exists(out) and os.path.getmtime(out) >= _deps_mtime(srcs):
        return f"{name}: up to date"
    cmd = [nvcc(), *ARCH, *FLAGS, "-o", out + ".tmp", *srcs]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {name}:\n{' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    os.replace(out + ".tmp", out)
    return f"{name}: built"


def build(force: bool = False) -> list[str]:
    for out in TARGETS:
        os.makedirs(os.path.dirname(out), exist_ok=True)
    with ThreadPoolExecutor(len(TARGETS)) as ex:
        futs = [ex.submit(_build_one, n, s, force) for n, s in TARGETS.items()]
        return [f.result() for f in futs]


if __name__ == "__main__":
    for line in build(force="--force" in sys.argv):
        print(line)
