"""NVFP4 x NVFP4 GEMM for B200 (sm_100a), drop-in for the nvfp4_gemm_cute package API.

gemm: C = alpha * dequant(A) @ dequant(B).T with per-shape launch configurations.
quantize_nvfp4 / dequantize_nvfp4 / swizzle_sf: NVFP4 packing in the layout the kernel reads,
computed by CUDA kernels bit-exact with the reference quantiser.
persisting_l2: scoped persisting-L2 limit for presets with persist_mb > 0.
nvfp4_linear / quantize_nvfp4_act: the LLM-projection call (activation quantised per call, weight
streamed by the skinny-M kernel with programmatic dependent launch); B200 additions.
"""

__version__ = "0.1.0"
from .api import device_status, gemm, persisting_l2, supported
from .presets import DEFAULT, PRESETS, Config, config_for
from .linear import nvfp4_linear
from .quant import (
    dequantize_nvfp4,
    quantize_nvfp4,
    quantize_nvfp4_act,
    quantize_nvfp4_global,
    swizzle_sf,
    tensor_amax,
)

__all__ = [
    "DEFAULT",
    "PRESETS",
    "Config",
    "config_for",
    "dequantize_nvfp4",
    "device_status",
    "gemm",
    "nvfp4_linear",
    "persisting_l2",
    "quantize_nvfp4",
    "quantize_nvfp4_act",
    "quantize_nvfp4_global",
    "supported",
    "swizzle_sf",
    "tensor_amax",
]
