"""LLM-projection call y = x . W^T on NVFP4 weights, with the activation quantised per call.

The reference quantises activations with quantize_nvfp4 and calls gemm (nvfp4_gemm_cute/api.py
and quant.py, global-scale recipe of docs/usage.md:14); it has no skinny-M kernel. Here, for up to
128 rows of x, the call is three launches on the current stream, each allowed to start before
the previous one ends (programmatic dependent launch):

1. quant.quantize_nvfp4_act: per-CTA partial maxima of |x|, then the quantiser, which derives
   gs_x = 6 * 448 / amax and alpha = 1 / (gs_x * gs_w) and writes the codes and swizzled scales.
2. The weight-streaming GEMM (tile (128, 128)) in the mode that streams W and its scales without
   waiting and loads x's codes, scales and alpha once step 1 has finished: the weight stream
   from HBM, which sets the call's time, starts while the activations are being quantised.

Larger x goes through the same activation quantiser and the regular gemm preset. The result
equals quantize_nvfp4_global(x) followed by gemm(...) with alpha = 1 / (gs_x * gs_w), bit for
bit.
"""

import torch

from . import api, presets
from .quant import quantize_nvfp4_act


def nvfp4_linear(x, weight, weight_sf, weight_gs, out=None, out_dtype=torch.bfloat16):
    """y = x . dequant(W)^T for x [M, K] (BF16/FP16/FP32) and NVFP4 weights W [N, K/2].

    Args:
        x: activations, quantised on the GPU in this call with their tensor-wide global scale.
        weight, weight_sf: packed W and its swizzled scales (quantize_nvfp4_global on W).
        weight_gs: W's global encode scale (one-element float32 CUDA tensor). W must not be
            written by the kernel that runs just before this call on the stream.
        out: optional [M, N] output of out_dtype.
    """
    m, k = x.shape
    if weight.shape[1] * 2 != k:
        raise ValueError(f"K mismatch: x is [{m}, {k}], weight is [{weight.shape[0]}, {weight.shape[1]}] packed")
    if m <= presets.STREAM_MAX_M:
        xq, xsf, _, alpha = quantize_nvfp4_act(x, weight_gs)
        return api._gemm(xq, weight, xsf, weight_sf, alpha, out, out_dtype, presets.SKINNY, 2)
    xq, xsf, _, alpha = quantize_nvfp4_act(x, weight_gs)
    return api.gemm(xq, weight, xsf, weight_sf, alpha=alpha, out=out, out_dtype=out_dtype)
