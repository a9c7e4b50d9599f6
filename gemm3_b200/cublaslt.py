"""The same NVFP4 GEMM through cuBLASLt on this GPU (libgemm3_b200_cublaslt.so).

A vendor baseline for bench.py and a second implementation that the GPU tests compare the
tcgen05 kernel with (the reference compares against cuBLASLt the same way,
benchmarks/compare.py:45-58). gemm3_b200.gemm never calls it.
"""

import ctypes
import os
import threading

import torch

from .build import CUBLASLT_LIB_PATH

EXPORTED_SYMBOLS = ("nvfp4_cublaslt_gemm", "nvfp4_cublaslt_last_status")
WORKSPACE_BYTES = 32 << 20

_lock = threading.Lock()
_lib = None
_workspace = {}
_OUT = {torch.float16: 0, torch.bfloat16: 1}


def lib():
    """Load the adapter once; RuntimeError if it was not built (the toolkit had no cuBLASLt)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(CUBLASLT_LIB_PATH):
                raise RuntimeError(f"{CUBLASLT_LIB_PATH} is missing; build it with `python -m gemm3_b200.build`")
            h = ctypes.CDLL(CUBLASLT_LIB_PATH)
            vp, i64 = ctypes.c_void_p, ctypes.c_int64
            h.nvfp4_cublaslt_gemm.restype = ctypes.c_int
            h.nvfp4_cublaslt_gemm.argtypes = [vp, vp, vp, vp, vp, ctypes.c_float, i64, i64, i64, ctypes.c_int32, vp,
                                              i64, vp]
            h.nvfp4_cublaslt_last_status.restype = ctypes.c_int32
            h.nvfp4_cublaslt_last_status.argtypes = []
            _lib = h
    return _lib


def gemm_cublaslt(a, b, a_sf, b_sf, alpha=1.0, out=None, out_dtype=torch.float16):
    """alpha * dequant(a) @ dequant(b).T by cuBLASLt; same operands as gemm3_b200.gemm.

    alpha is taken as a host float (a one-element tensor is read back, which synchronises).
    """
    m, half_k = a.shape
    n, k = b.shape[0], 2 * half_k
    if out_dtype not in _OUT:
        raise ValueError(f"unsupported output dtype {out_dtype}")
    if isinstance(alpha, torch.Tensor):
        alpha = float(alpha.reshape(-1)[0].item())
    dev = a.device
    if out is None:
        out = torch.empty(m, n, dtype=out_dtype, device=dev)
    ws = _workspace.get(dev)
    if ws is None:
        ws = _workspace[dev] = torch.empty(WORKSPACE_BYTES, dtype=torch.uint8, device=dev)
    with torch.cuda.device(dev):
        rc = lib().nvfp4_cublaslt_gemm(
            a.data_ptr(), b.data_ptr(), a_sf.data_ptr(), b_sf.data_ptr(), out.data_ptr(), float(alpha), m, n, k,
            _OUT[out_dtype], ws.data_ptr(), ws.numel(), torch.cuda.current_stream(dev).cuda_stream,
        )
    if rc != 0:
        raise RuntimeError(f"nvfp4_cublaslt_gemm failed: status {rc}, cuBLAS status {lib().nvfp4_cublaslt_last_status()}")
    return out
