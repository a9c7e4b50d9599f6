"""Device properties the B200 GEMM is launched on (nvfp4_gemm_cute/hw.py:8-28)."""

import ctypes
import functools

import torch

from . import _lib


@functools.cache
def get_max_active_clusters(cluster_size: int) -> int:
    """Return how many clusters of cluster_size CTAs of the GEMM kernel fit on the current GPU.

    The kernel is the one gemm() launches by default, the CTA-pair kernel (tile (256, 256)); with
    cluster_size 2 the answer is the number of CTA pairs its persistent grid holds (74 on a B200
    whose 148 SMs all pair up).

    Uses cudaOccupancyMaxActiveClusters through the extension; if the occupancy query fails it
    falls back to the SM count divided by the cluster size, like the reference.
    """
    torch.cuda.init()
    out = ctypes.c_int32(0)
    _lib.check(_lib.lib().nvfp4_max_active_clusters(int(cluster_size), ctypes.byref(out)),
               "nvfp4_max_active_clusters")
    return int(out.value)


def arch() -> str:
    """Return the compute architecture of the current CUDA device, such as "sm_100"."""
    major, minor = torch.cuda.get_device_capability()
    return f"sm_{major}{minor}"


@functools.cache
def device_info(device: int):
    """(sm_count, (major, minor), l2_bytes) of a CUDA device, from the extension."""
    sm, ma, mi, l2 = ctypes.c_int32(), ctypes.c_int32(), ctypes.c_int32(), ctypes.c_int64()
    _lib.check(
        _lib.lib().nvfp4_device_info(int(device), ctypes.byref(sm), ctypes.byref(ma), ctypes.byref(mi),
                                     ctypes.byref(l2)),
        "nvfp4_device_info",
    )
    return int(sm.value), (int(ma.value), int(mi.value)), int(l2.value)
