"""numpy/ctypes front end of the CPU oracle (nvfp4_oracle.c).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and bench.py's cpu_baseline
leg as the checker; the gemm3_b200 package never imports it.

Functions follow nvfp4_gemm_cute/quant.py and testing.py of the reference:
  quantize      quant.py:41-59      swizzle      quant.py:31-38
  dequantize    quant.py:62-70      gemm_fp64    testing.py:18-27 (dequantised matmul, in FP64)
  reference_fp32  testing.py:18-27  (FP32 dequantised matmul, as the reference's own check)
"""

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "nvfp4_oracle.c")
LIB = os.path.join(HERE, "_build", "liboracle.so")
CFLAGS = ["-O2", "-fopenmp", "-ffp-contract=off", "-fno-fast-math", "-fPIC", "-shared", "-std=c11"]

_lib = None


def build(force=False):
    """Compile the C restatement (gcc, OpenMP) into oracle/_build/."""
    if not force and os.path.exists(LIB) and os.path.getmtime(LIB) >= os.path.getmtime(SRC):
        return LIB
    os.makedirs(os.path.dirname(LIB), exist_ok=True)
    tmp = LIB + ".tmp"
    subprocess.run(["gcc", *CFLAGS, "-o", tmp, SRC, "-lm"], check=True)
    os.replace(tmp, LIB)
    return LIB


def lib():
    global _lib
    if _lib is None:
        build()
        L = ctypes.CDLL(LIB)
        vp, i64, f32, i32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_float, ctypes.c_int
        L.oracle_quantize.argtypes = [vp, i64, i64, f32, i32, vp, vp]
        L.oracle_swizzle.argtypes = [vp, i64, i64, vp]
        L.oracle_dequantize.argtypes = [vp, vp, i64, i64, f32, i32, vp]
        L.oracle_e4m3_encode_n.argtypes = [vp, i64, vp]
        L.oracle_e2m1_code_n.argtypes = [vp, i64, vp]
        L.oracle_num_threads.restype = ctypes.c_int
        for f in ("oracle_quantize", "oracle_swizzle", "oracle_dequantize", "oracle_e4m3_encode_n",
                  "oracle_e2m1_code_n"):
            getattr(L, f).restype = None
        _lib = L
    return _lib


def _ptr(a):
    return a.ctypes.data_as(ctypes.c_void_p)


def num_threads():
    return int(lib().oracle_num_threads())


def e4m3_encode(x):
    x = np.ascontiguousarray(x, dtype=np.float32).ravel()
    out = np.empty(x.size, dtype=np.uint8)
    lib().oracle_e4m3_encode_n(_ptr(x), x.size, _ptr(out))
    return out


def e2m1_code(x):
    x = np.ascontiguousarray(x, dtype=np.float32).ravel()
    out = np.empty(x.size, dtype=np.uint8)
    lib().oracle_e2m1_code_n(_ptr(x), x.size, _ptr(out))
    return out


def swizzle(sf_lin):
    sf_lin = np.ascontiguousarray(sf_lin, dtype=np.uint8)
    rows, cols = sf_lin.shape
    out = np.empty(-(-rows // 128) * 128 * (-(-cols // 4)) * 4, dtype=np.uint8)
    lib().oracle_swizzle(_ptr(sf_lin), rows, cols, _ptr(out))
    return out


def quantize(x, global_scale=1.0, div_mode=1):
    """(packed [rows, K/2], sf_swizzled flat, sf_linear [rows, K/16]) of a [rows, K] array.

    div_mode 1 reproduces the reference run on CPU tensors, 0 on CUDA tensors.
    """
    x = np.ascontiguousarray(x, dtype=np.float32)
    rows, k = x.shape
    assert k % 16 == 0, "K must be a multiple of 16"
    packed = np.empty((rows, k // 2), dtype=np.uint8)
    sf_lin = np.empty((rows, k // 16), dtype=np.uint8)
    lib().oracle_quantize(_ptr(x), rows, k, float(np.float32(global_scale)), int(div_mode), _ptr(packed),
                          _ptr(sf_lin))
    return packed, swizzle(sf_lin), sf_lin


def dequantize(packed, sf_lin, global_scale=1.0, div_mode=1):
    packed = np.ascontiguousarray(packed, dtype=np.uint8)
    sf_lin = np.ascontiguousarray(sf_lin, dtype=np.uint8)
    rows, kp = packed.shape
    out = np.empty((rows, kp * 2), dtype=np.float32)
    lib().oracle_dequantize(_ptr(packed), _ptr(sf_lin), rows, kp * 2, float(np.float32(global_scale)),
                            int(div_mode), _ptr(out))
    return out


def gemm_fp64(a_packed, a_sf_lin, b_packed, b_sf_lin, alpha=1.0):
    """alpha * dequant(A) @ dequant(B).T in float64 (the dequantised values are exact in FP32)."""
    a = dequantize(a_packed, a_sf_lin).astype(np.float64)
    b = dequantize(b_packed, b_sf_lin).astype(np.float64)
    return float(alpha) * (a @ b.T)


def reference_fp32(a_packed, a_sf_lin, b_packed, b_sf_lin):
    """FP32 dequantised matmul, the reference's acceptance oracle."""
    a = dequantize(a_packed, a_sf_lin)
    b = dequantize(b_packed, b_sf_lin)
    return a @ b.T
