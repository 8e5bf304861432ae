"""Build libfme_cuda.so in-tree with nvcc for sm_100a (B200).

    python fast-mario-env_b200/build.py          # or __graft_entry__.build()

The library is a plain C-ABI shared object (no Python extension, no JIT): FMA contraction is disabled so the
INTER_AREA float arithmetic keeps OpenCV's exact operation order.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libfme_cuda.so")
SOURCES = ["fme.cu"]
DEPS = ["fme.cu", "fme_kernels.cuh", "fme_core.h", "fme_agent.h", "fme_render.h", "fme_defs.h", "fme_tables.h", "fme_fast.h", "fme_dp.h", "fme_ppo.cuh", "fme_replay.cuh"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found (set NVCC)")


def command(out: str = LIB, extra=()) -> list[str]:
    inc = os.path.join(os.path.dirname(HERE), "include")
    return [nvcc_path(), *ARCH, "-O3", "-lineinfo", "-std=c++17", "--fmad=false", "-Xptxas", "-v",
            "-Xcompiler", "-fPIC", "-shared", "-I", inc, "-I", CSRC, *extra,
            *[os.path.join(CSRC, s) for s in SOURCES], "-o", out]


def up_to_date(out: str = LIB) -> bool:
    if not os.path.exists(out):
        return False
    t = os.path.getmtime(out)
    deps = [os.path.join(CSRC, d) for d in DEPS] + [os.path.join(os.path.dirname(HERE), "include", "fme.h")]
    return all(os.path.getmtime(d) <= t for d in deps if os.path.exists(d))


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and up_to_date():
        return LIB
    cmd = command()
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError("nvcc failed building libfme_cuda.so")
    if verbose:
        sys.stderr.write(r.stderr)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True)
    print(LIB)
