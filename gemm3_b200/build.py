"""Build libgemm3_b200.so in-tree with nvcc for sm_100a.

python -m gemm3_b200.build [--verbose]

The library links the CUDA runtime statically and resolves driver entry points at run time, so it
loads (and its symbols can be inspected) on a machine without a GPU or driver.
"""

import os
import shutil
import subprocess
import sys

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
REPO_DIR = os.path.dirname(PKG_DIR)
CSRC = os.path.join(PKG_DIR, "csrc")
LIB_NAME = "libgemm3_b200.so"
LIB_PATH = os.path.join(PKG_DIR, LIB_NAME)
SOURCES = [os.path.join(CSRC, "capi.cu")]
DEPENDS = SOURCES + [
    os.path.join(CSRC, f) for f in ("ptx.cuh", "gemm_kernel.cuh", "gemm_pair_kernel.cuh", "quant_kernel.cuh")
] + [os.path.join(REPO_DIR, "include", "nvfp4_gemm.h")]

NVCC_FLAGS = [
    "-gencode",
    "arch=compute_100a,code=sm_100a",
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "-Xcompiler",
    "-fPIC",
    "-shared",
    "-cudart",
    "static",
]


def nvcc_path():
    for cand in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found; the CUDA toolkit is required to build gemm3_b200")


def up_to_date():
    if not os.path.exists(LIB_PATH):
        return False
    t = os.path.getmtime(LIB_PATH)
    return all(os.path.getmtime(f) <= t for f in DEPENDS)


def build(force=False, verbose=False):
    """Compile the extension unless it is newer than every source. Returns the library path."""
    if not force and up_to_date():
        return LIB_PATH
    tmp = LIB_PATH + ".tmp"
    cmd = [nvcc_path(), *NVCC_FLAGS, "-o", tmp, *SOURCES]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=not verbose, text=True)
    if res.returncode != 0:
        msg = (res.stderr or "") + (res.stdout or "")
        raise RuntimeError(f"nvcc failed ({res.returncode}):\n{msg}")
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="--verbose" in sys.argv))
