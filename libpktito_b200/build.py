"""Builds libpktito_b200.so in place: the sm_100a kernels, the C ABI and the
cuda-b200 backend table, with nvcc and the host C compiler.

    python -m libpktito_b200.build        (or libpktito_b200.build.build())

The float code is compiled without any contraction or fast-math: -fmad=false
-prec-div=true -prec-sqrt=true -ftz=false for the device, and
-ffp-contract=off for the host C, the reference's own rule (its Makefile
builds every backend with -ffp-contract=off), so every operation rounds
where the source says it does.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libpktito_b200.so")

CU_SOURCES = ["pkb_api.cu", "pkb_host.cu", "pkb_gemm.cu", "pkb_quantize.cu", "pkb_noalloc.cu", "pkb_selftest.cu", "pkb_fused.cu",
              "pkb_attn.cu", "pkb_tdt.cu"]
C_SOURCES = ["cuda_b200.c"]

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xptxas", "-v",
    "-fmad=false", "-prec-div=true", "-prec-sqrt=true", "-ftz=false",
    "--expt-relaxed-constexpr", "-I" + os.path.join(ROOT, "include"),
]
CC_FLAGS = ["-O2", "-std=c11", "-fPIC", "-ffp-contract=off", "-fno-math-errno", "-Wall", "-Wextra",
            "-I" + os.path.join(ROOT, "include")]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _run(cmd: list[str], log: list[str]) -> None:
    r = subprocess.run(cmd, capture_output=True, text=True)
    log.append(" ".join(cmd) + "\n" + r.stdout + r.stderr)
    if r.returncode != 0:
        raise RuntimeError("build step failed:\n" + " ".join(cmd) + "\n" + r.stdout + r.stderr)


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(force: bool = False, verbose: bool = False) -> str:
    """Compile every source for sm_100a and link libpktito_b200.so; returns its path."""
    os.makedirs(BUILD, exist_ok=True)
    nvcc = _nvcc()
    headers = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".h", ".cuh"))]
    headers += [os.path.join(ROOT, "include", f) for f in os.listdir(os.path.join(ROOT, "include"))]
    objs, log = [], []
    for src in CU_SOURCES:
        s = os.path.join(CSRC, src)
        o = os.path.join(BUILD, src + ".o")
        if force or _stale(o, [s] + headers):
            _run([nvcc, *ARCH, *NVCC_FLAGS, "-c", s, "-o", o], log)
        objs.append(o)
    cc = os.environ.get("CC", "gcc")
    for src in C_SOURCES:
        s = os.path.join(CSRC, src)
        o = os.path.join(BUILD, src + ".o")
        if force or _stale(o, [s] + headers):
            _run([cc, *CC_FLAGS, "-c", s, "-o", o], log)
        objs.append(o)
    if force or _stale(LIB, objs):
        _run([nvcc, *ARCH, "-shared", "-o", LIB, *objs, "-lcudart", "-Xlinker", "-soname=libpktito_b200.so"], log)
    with open(os.path.join(BUILD, "build.log"), "w") as f:
        f.write("\n".join(log))
    if verbose:
        print("\n".join(log))
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
