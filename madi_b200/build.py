"""Build libmadi_q8.so in-tree with nvcc for sm_100a.

The library is plain C-ABI (include/madi_q8.h) with the CUDA runtime linked
statically, so any process can load it: the Python host layer through ctypes,
a Zig host through @cImport, a C/C++ program through the header.

    python -m madi_b200.build [--verbose]
"""
import argparse
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
BUILD = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "libmadi_q8.so")
SOURCES = ["runtime.cu", "q8_gemv.cu", "q8_gemv_tile.cu", "q8_gemm_tc.cu", "q8_misc.cu", "res_ln.cu", "decode_step.cu", "attn.cu", "flash_enc.cu", "xchg.cu"]
HEADERS = ["common.cuh", "internal.h"]

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
              "-I", os.path.join(ROOT, "include")]


def nvcc() -> str:
    cand = os.environ.get("NVCC") or shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand) and not shutil.which(cand):
        raise RuntimeError("nvcc not found; the madi_b200 CUDA library cannot be built")
    return cand


def _stale(target: str, deps) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(verbose: bool = False, force: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    hdrs = [os.path.join(CSRC, h) for h in HEADERS] + [os.path.join(ROOT, "include", "madi_q8.h")]
    objs = []
    for src in SOURCES:
        s = os.path.join(CSRC, src)
        o = os.path.join(BUILD, src.replace(".cu", ".o"))
        objs.append(o)
        if force or _stale(o, [s] + hdrs + [__file__]):
            cmd = [nvcc()] + ARCH + NVCC_FLAGS + ["-c", s, "-o", o]
            if verbose:
                cmd += ["-Xptxas", "-v"]
                print(" ".join(cmd), flush=True)
            subprocess.run(cmd, check=True)
    if force or _stale(LIB, objs):
        cmd = [nvcc()] + ARCH + ["-shared", "-o", LIB] + objs + ["-lpthread"]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args()
    print(build(verbose=a.verbose, force=a.force))
    sys.exit(0)
