"""Builds libxksv_cuda.so (sm_100a) in-tree with nvcc.

    python xks-vectorforge_b200/build.py [--verbose]

The library has no Python or torch dependency: it is a plain C-ABI shared
object (include/xksv_cuda.h) that ctypes, cgo or C++ callers load directly.
"""
import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent
CSRC = HERE / "csrc"
LIB = HERE / "libxksv_cuda.so"
SOURCES = ["api.cu", "parallel_kernels.cu", "serial_kernels.cu", "raw_kernels.cu", "pack_host.cpp", "noalloc.cu",
           "tp.cpp", "tc_gemm.cu", "fused_gemm.cu", "sha256.cu", "pack_gpu.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc():
    cand = os.environ.get("NVCC") or "/usr/local/cuda/bin/nvcc"
    return cand if Path(cand).exists() else "nvcc"


def build(verbose=False, force=False):
    srcs = [CSRC / s for s in SOURCES]
    deps = srcs + list(CSRC.glob("*.h")) + list(CSRC.glob("*.cuh")) + [ROOT / "include" / "xksv_cuda.h"]
    if LIB.exists() and not force and all(LIB.stat().st_mtime >= d.stat().st_mtime for d in deps):
        return LIB
    cmd = [nvcc(), *ARCH, "-O3", "-lineinfo", "-std=c++17", "-shared", "-Xcompiler", "-fPIC,-pthread",
           "-I", str(ROOT / "include"), "-o", str(LIB) + ".tmp", *map(str, srcs), "-ldl"]
    if verbose:
        cmd[1:1] = ["-Xptxas", "-v"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError("nvcc failed building libxksv_cuda.so")
    if verbose:
        sys.stderr.write(r.stderr)
    os.replace(str(LIB) + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    build(verbose="--verbose" in sys.argv, force=True)
    print(LIB)
