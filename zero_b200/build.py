"""Build libzgpu.so in-tree: hand-written CUDA for sm_100a plus the C++ host runtime.

Run as ``python zero_b200/build.py`` (or through ``__graft_entry__.build()``);
it does not import the package, which needs the library this script builds.
Objects go to ``zero_b200/_build/``; the shared library lands next to this
file so that it travels with the source tree.
"""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
BUILD = HERE / "_build"
LIB = HERE / "libzgpu.so"
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
CUDA_FLAGS = ARCH + [
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "-Xcompiler",
    "-fPIC,-O2,-Wall",
    "--expt-relaxed-constexpr",
]
CXX_FLAGS = ["-O2", "-fPIC", "-std=c++17", "-Wall", "-pthread"]
# ZGPU_DEVICE_CHECKS=1 builds kernels that bounds-check their shared/global
# accesses, record the first failure in the status block and skip it.
if os.environ.get("ZGPU_DEVICE_CHECKS") == "1":
    CUDA_FLAGS.append("-DZGPU_DEVICE_CHECKS")
# ZGPU_STEP_TRACE=1 records the persistent kernel's stage timeline (CTA 0)
# and exports zgpu_debug_step_trace to read it.
if os.environ.get("ZGPU_STEP_TRACE") == "1":
    CUDA_FLAGS.append("-DZGPU_STEP_TRACE")

CU_SOURCES = ["gemv.cu", "attention.cu", "attention_static.cu", "step.cu", "ops.cu", "moe.cu", "mla.cu", "mma_gemm.cu", "digit_mma.cu", "prefill.cu", "sampler.cu", "kquant.cu", "mha.cu",
              "ctx.cu", "model.cu", "ds2.cu"]
CXX_SOURCES = ["synth.cpp", "smodel.cpp", "detok.cpp"]


def _run(cmd: list[str]) -> None:
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        sys.stderr.write(" ".join(cmd) + "\n" + proc.stdout + proc.stderr)
        raise RuntimeError(f"build step failed: {cmd[0]} {cmd[-1]}")
    if proc.stderr.strip():
        sys.stderr.write(proc.stderr)


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def build(verbose_ptxas: bool = False, force: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    headers = list(CSRC.glob("*.h")) + list(CSRC.glob("*.cuh")) + [HERE.parent / "include" / "zgpu.h"]
    objs: list[Path] = []
    for src in CU_SOURCES:
        s = CSRC / src
        o = BUILD / (src + ".o")
        if force or _stale(o, [s] + headers):
            cmd = [NVCC] + CUDA_FLAGS + (["-Xptxas", "-v"] if verbose_ptxas else []) + ["-c", str(s), "-o", str(o)]
            _run(cmd)
        objs.append(o)
    for src in CXX_SOURCES:
        s = CSRC / src
        o = BUILD / (src + ".o")
        if force or _stale(o, [s] + headers):
            _run(["g++"] + CXX_FLAGS + ["-c", str(s), "-o", str(o)])
        objs.append(o)
    if force or _stale(LIB, objs):
        _run([NVCC] + ARCH + ["-shared", "-o", str(LIB)] + [str(o) for o in objs] + ["-lpthread"])
    return LIB


if __name__ == "__main__":
    build(verbose_ptxas="-v" in sys.argv, force="-f" in sys.argv)
    print(LIB)
