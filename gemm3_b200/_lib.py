"""ctypes binding of libgemm3_b200.so (the C ABI declared in include/nvfp4_gemm.h).

The library is the only compute path: if it is missing or fails to load, every operation raises.
"""

import ctypes
import os
import threading

from .build import LIB_PATH

# nvfp4_status values (include/nvfp4_gemm.h)
OK = 0
ERR_INVALID_VALUE = 1
ERR_MISALIGNED = 2
ERR_UNSUPPORTED = 3
ERR_CUDA = 4
ERR_TENSOR_MAP = 5
ERR_TOO_LARGE = 6

NOALLOC_MAX_ELEMENTS = 1 << 31
ACT_WORKSPACE_BYTES = 4096
MAX_GATHER_DST = 8
IPC_HANDLE_BYTES = 64

DTYPE_F16, DTYPE_BF16, DTYPE_F32 = 0, 1, 2
L2_NORMAL, L2_EVICT_FIRST, L2_EVICT_LAST = 0, 1, 2

EXPORTED_SYMBOLS = (
    "nvfp4_gemm_run",
    "nvfp4_quantize",
    "nvfp4_amax",
    "nvfp4_dequantize",
    "nvfp4_swizzle_sf",
    "nvfp4_max_active_clusters",
    "nvfp4_device_info",
    "nvfp4_set_persisting_l2",
    "nvfp4_strerror",
    "nvfp4_last_cuda_error",
    "nvfp4_abi_version",
    "nvfp4_quantize_global_noalloc",
    "nvfp4_selftest_wait_timeout",
    "nvfp4_quantize_act",
    "nvfp4_gemm_run_gather",
    "nvfp4_ipc_get_handle",
    "nvfp4_ipc_open",
    "nvfp4_ipc_close",
)


class GemmConfig(ctypes.Structure):
    """Mirror of struct nvfp4_gemm_config."""

    _fields_ = [
        ("struct_size", ctypes.c_int32),
        ("tile_m", ctypes.c_int32),
        ("tile_n", ctypes.c_int32),
        ("raster_band", ctypes.c_int32),
        ("raster_along_m", ctypes.c_int32),
        ("l2_policy_a", ctypes.c_int32),
        ("l2_policy_b", ctypes.c_int32),
        ("l2_policy_sfa", ctypes.c_int32),
        ("l2_policy_sfb", ctypes.c_int32),
        ("store_evict_first", ctypes.c_int32),
        ("epi_store_pace_ns", ctypes.c_int32),
        ("tma_b_first", ctypes.c_int32),
        ("max_ctas", ctypes.c_int32),
        ("pdl", ctypes.c_int32),
    ]


_lock = threading.Lock()
_lib = None

_vp, _i32, _i64, _f32 = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_float
_SIGNATURES = {
    "nvfp4_gemm_run": (
        ctypes.c_int,
        [_vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i32, ctypes.POINTER(GemmConfig), _vp, _vp],
    ),
    "nvfp4_quantize": (
        ctypes.c_int,
        [_vp, _i32, _i64, _i64, _f32, _vp, _i32, _i32, _vp, _vp, _vp, _vp, _vp],
    ),
    "nvfp4_amax": (ctypes.c_int, [_vp, _i32, _i64, _vp, _vp]),
    "nvfp4_dequantize": (ctypes.c_int, [_vp, _vp, _i64, _i64, _f32, _i32, _vp, _vp]),
    "nvfp4_swizzle_sf": (ctypes.c_int, [_vp, _i64, _i64, _vp, _vp]),
    "nvfp4_max_active_clusters": (ctypes.c_int, [_i32, ctypes.POINTER(_i32)]),
    "nvfp4_device_info": (
        ctypes.c_int,
        [_i32, ctypes.POINTER(_i32), ctypes.POINTER(_i32), ctypes.POINTER(_i32), ctypes.POINTER(_i64)],
    ),
    "nvfp4_set_persisting_l2": (ctypes.c_int, [_i64, ctypes.POINTER(_i64)]),
    "nvfp4_strerror": (ctypes.c_char_p, [_i32]),
    "nvfp4_last_cuda_error": (_i32, []),
    "nvfp4_abi_version": (_i32, []),
    "nvfp4_quantize_global_noalloc": (ctypes.c_int, [_vp, _i32, _i64, _i64, _vp, _vp, _vp, _vp, _vp]),
    "nvfp4_selftest_wait_timeout": (ctypes.c_int, [_vp, _i32, _vp]),
    "nvfp4_quantize_act": (ctypes.c_int, [_vp, _i32, _i64, _i64, _vp, _vp, _vp, _vp, _vp, _vp, _vp]),
    "nvfp4_gemm_run_gather": (
        ctypes.c_int,
        [_vp, _vp, _vp, _vp, ctypes.POINTER(_vp), _i32, _i64, _i64, _vp, _i64, _i64, _i64, _i32,
         ctypes.POINTER(GemmConfig), _vp, _vp],
    ),
    "nvfp4_ipc_get_handle": (ctypes.c_int, [_vp, _vp, ctypes.POINTER(_i64)]),
    "nvfp4_ipc_open": (ctypes.c_int, [_vp, _i64, ctypes.POINTER(_vp)]),
    "nvfp4_ipc_close": (ctypes.c_int, [_vp, _i64]),
}


def lib():
    """Load the extension once. Raises RuntimeError if it has not been built or cannot load."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise RuntimeError(
                    f"{LIB_PATH} is missing; build it with `python -m gemm3_b200.build` "
                    "(there is no fallback implementation)"
                )
            handle = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in _SIGNATURES.items():
                fn = getattr(handle, name)
                fn.restype = res
                fn.argtypes = args
            _lib = handle
    return _lib


def check(rc, what):
    """Turn a non-zero nvfp4_status into an exception (ValueError for bad arguments)."""
    if rc == OK:
        return
    L = lib()
    text = L.nvfp4_strerror(rc).decode()
    if rc == ERR_CUDA:
        text += f" (cudaError {L.nvfp4_last_cuda_error()})"
    if rc in (ERR_INVALID_VALUE, ERR_MISALIGNED):
        raise ValueError(f"{what}: {text}")
    raise RuntimeError(f"{what} failed: {text} [status {rc}]")
