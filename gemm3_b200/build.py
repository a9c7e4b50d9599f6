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
    os.path.join(CSRC, f) for f in ("ptx.cuh", "gemm_kernel.cuh", "gemm_pair_kernel.cuh", "gemm_stream_kernel.cuh", "quant_kernel.cuh")
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


# The cuBLASLt adapter (vendor baseline, not on the compute path): a separate library that links
# the toolkit's libcublasLt, found at run time through this rpath or an already loaded copy.
CUBLASLT_LIB_PATH = os.path.join(PKG_DIR, "libgemm3_b200_cublaslt.so")
CUBLASLT_SOURCES = [os.path.join(CSRC, "cublaslt_adapter.cu")]
CUBLASLT_DEPENDS = CUBLASLT_SOURCES + [os.path.join(REPO_DIR, "include", "nvfp4_cublaslt.h")]


def _cuda_root():
    return os.path.dirname(os.path.dirname(os.path.realpath(nvcc_path())))


def up_to_date(path=LIB_PATH, depends=DEPENDS):
    if not os.path.exists(path):
        return False
    t = os.path.getmtime(path)
    return all(os.path.getmtime(f) <= t for f in depends)


def _compile(path, sources, extra, verbose):
    tmp = path + ".tmp"
    cmd = [nvcc_path(), *NVCC_FLAGS, "-o", tmp, *sources, *extra]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=not verbose, text=True)
    if res.returncode != 0:
        msg = (res.stderr or "") + (res.stdout or "")
        raise RuntimeError(f"nvcc failed ({res.returncode}):\n{msg}")
    os.replace(tmp, path)


def build_cublaslt(force=False, verbose=False):
    """Compile the cuBLASLt adapter if the toolkit has cuBLASLt. Returns its path, or None."""
    root = _cuda_root()
    lib_dir = os.path.join(root, "lib64")
    if not os.path.exists(os.path.join(root, "include", "cublasLt.h")):
        return None
    if force or not up_to_date(CUBLASLT_LIB_PATH, CUBLASLT_DEPENDS):
        _compile(CUBLASLT_LIB_PATH, CUBLASLT_SOURCES, [f"-L{lib_dir}", "-lcublasLt", f"-Xlinker=-rpath,{lib_dir}"],
                 verbose)
    return CUBLASLT_LIB_PATH


def build(force=False, verbose=False):
    """Compile the extension (and the cuBLASLt adapter) unless newer than every source. Returns
    the extension's path."""
    if force or not up_to_date():
        _compile(LIB_PATH, SOURCES, [], verbose)
    build_cublaslt(force, verbose)
    return LIB_PATH


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="--verbose" in sys.argv))
