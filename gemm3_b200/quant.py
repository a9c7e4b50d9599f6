"""NVFP4 quantisation in the layout the GEMM consumes, computed by CUDA kernels.

Same functions and format as nvfp4_gemm_cute/quant.py: E2M1 values with one E4M3 scale per 16
consecutive elements along K, two values per byte (element 2j in the low nibble), and scale
factors handed to the GEMM in the 128x4 swizzled layout (rows padded to 128 and scale columns to
4, each (128 rows, 4 columns) tile stored as [32][4][4] = (row % 32, row // 32, column)).

The kernels reproduce the reference's FP32 arithmetic bit for bit. Where PyTorch itself rounds
differently on CPU and on CUDA (a division by a Python scalar is a true division on CPU and a
multiplication by the FP32 reciprocal on CUDA), the result follows the device of the input
tensor, so a call returns exactly what the reference returns for the same tensor. CPU tensors
are processed on the current CUDA device and the results copied back; there is no CPU
implementation.
"""

import torch

from . import _lib

SF_VEC = 16

_IN_DTYPES = {torch.float16: _lib.DTYPE_F16, torch.bfloat16: _lib.DTYPE_BF16, torch.float32: _lib.DTYPE_F32}


def _stream(dev):
    return torch.cuda.current_stream(dev).cuda_stream


def _cuda_device(t):
    if t.device.type == "cuda":
        return t.device
    if not torch.cuda.is_available():
        raise RuntimeError("gemm3_b200 quantisation runs on a CUDA device; none is available")
    return torch.device("cuda", torch.cuda.current_device())


def sf_swizzled_size(rows: int, k: int) -> int:
    """Bytes of the 128x4 swizzled scale layout for a [rows, k] operand."""
    return -(-rows // 128) * 128 * (-(-(k // SF_VEC) // 4)) * 4


def swizzle_sf(sf):
    """Convert [rows, cols] E4M3 scale factors (as uint8) to the 128x4 swizzled layout (flat)."""
    rows, cols = sf.shape
    home = sf.device
    dev = _cuda_device(sf)
    src = sf.view(torch.uint8).to(dev).contiguous()
    out = torch.empty(-(-rows // 128) * 128 * (-(-cols // 4)) * 4, dtype=torch.uint8, device=dev)
    with torch.cuda.device(dev):
        rc = _lib.lib().nvfp4_swizzle_sf(src.data_ptr(), rows, cols, out.data_ptr(), _stream(dev))
    _lib.check(rc, "nvfp4_swizzle_sf")
    return out.to(home)


def _run_quantize(x, gs_value, gs_tensor, gs_mode, div_mode, want_gs=False):
    rows, k = x.shape
    assert k % SF_VEC == 0, "K must be a multiple of 16"
    dev = _cuda_device(x)
    src = x if x.dtype in _IN_DTYPES else x.float()
    src = src.to(dev).contiguous()
    packed = torch.empty(rows, k // 2, dtype=torch.uint8, device=dev)
    sf_swz = torch.empty(sf_swizzled_size(rows, k), dtype=torch.uint8, device=dev)
    sf_lin = torch.empty(rows, k // SF_VEC, dtype=torch.uint8, device=dev)
    gs_out = torch.empty(1, dtype=torch.float32, device=dev) if want_gs else None
    gs_ptr = gs_tensor.data_ptr() if gs_tensor is not None else None
    with torch.cuda.device(dev):
        rc = _lib.lib().nvfp4_quantize(
            src.data_ptr(), _IN_DTYPES[src.dtype], rows, k, float(gs_value), gs_ptr, gs_mode, div_mode,
            packed.data_ptr(), sf_swz.data_ptr(), sf_lin.data_ptr(),
            gs_out.data_ptr() if gs_out is not None else None, _stream(dev),
        )
    _lib.check(rc, "nvfp4_quantize")
    return packed, sf_swz, sf_lin, gs_out


def quantize_nvfp4(x, global_scale: float = 1.0):
    """Quantize a [rows, K] float tensor to NVFP4 (nvfp4_gemm_cute/quant.py:41-59).

    global_scale multiplies x before quantisation: a Python float, or a one-element float32 CUDA
    tensor (read on the device).

    Returns:
        (packed, sf_swizzled, sf_linear): packed is [rows, K/2] uint8; sf_swizzled is the flat
        128x4 layout the kernel reads; sf_linear is [rows, K/16] uint8 (E4M3 bits) for reference
        dequantization. Results live on x's device.
    """
    home = x.device
    div_mode = 0 if home.type == "cuda" else 1
    if isinstance(global_scale, torch.Tensor):
        gs_t = global_scale.reshape(1).to(device=_cuda_device(x), dtype=torch.float32)
        packed, sf_swz, sf_lin, _ = _run_quantize(x, 0.0, gs_t, 1, div_mode)
    else:
        packed, sf_swz, sf_lin, _ = _run_quantize(x, global_scale, None, 0, div_mode)
    return packed.to(home), sf_swz.to(home), sf_lin.to(home)


def tensor_amax(x):
    """max |x| as a one-element float32 tensor on x's CUDA device (NaN propagates)."""
    dev = _cuda_device(x)
    src = (x if x.dtype in _IN_DTYPES else x.float()).to(dev).contiguous()
    out = torch.empty(1, dtype=torch.float32, device=dev)
    with torch.cuda.device(dev):
        rc = _lib.lib().nvfp4_amax(src.data_ptr(), _IN_DTYPES[src.dtype], src.numel(), out.data_ptr(), _stream(dev))
    _lib.check(rc, "nvfp4_amax")
    return out


def quantize_nvfp4_global(x):
    """Quantize with a per-tensor FP32 global encode scale gs = 6 * 448 / amax(|x|).

    The amax and gs stay on the device (two kernel launches, no host synchronisation). gs is 1
    when amax is 0 or not finite.

    Returns:
        (packed, sf_swizzled, sf_linear, global_scale): global_scale is a one-element float32 CUDA
        tensor; the GEMM alpha for operands A and B is 1 / (gs_A * gs_B).
    """
    if x.device.type != "cuda":
        raise ValueError("quantize_nvfp4_global needs a CUDA tensor")
    amax = tensor_amax(x)
    packed, sf_swz, sf_lin, gs = _run_quantize(x, 0.0, amax, 2, 0, want_gs=True)
    return packed, sf_swz, sf_lin, gs


def dequantize_nvfp4(packed, sf_linear, global_scale: float = 1.0):
    """Expand packed NVFP4 plus linear scale factors back to a float32 [rows, K] tensor
    (nvfp4_gemm_cute/quant.py:62-70)."""
    rows, kp = packed.shape
    k = kp * 2
    home = packed.device
    dev = _cuda_device(packed)
    div_mode = 0 if home.type == "cuda" else 1
    p = packed.to(dev).contiguous()
    s = sf_linear.view(torch.uint8).to(dev).contiguous()
    if s.numel() != rows * (k // SF_VEC):
        raise ValueError(f"sf_linear has {s.numel()} entries, expected {rows * (k // SF_VEC)}")
    out = torch.empty(rows, k, dtype=torch.float32, device=dev)
    with torch.cuda.device(dev):
        rc = _lib.lib().nvfp4_dequantize(
            p.data_ptr(), s.data_ptr(), rows, k, float(global_scale), div_mode, out.data_ptr(), _stream(dev)
        )
    _lib.check(rc, "nvfp4_dequantize")
    return out.to(home)


def quantize_nvfp4_act(x, gs_other=None):
    """Quantize activations with their tensor-wide global scale, for an LLM projection call.

    Same result, bit for bit, as quantize_nvfp4_global(x) (without the linear scales). Two
    kernels chained by programmatic dependent launch: per-CTA partial maxima, then the
    quantiser, which also derives gs = 6 * 448 / amax and, if gs_other (a one-element float32
    CUDA tensor, e.g. the weight's global scale) is given, the GEMM alpha = 1 / (gs * gs_other).
    A weight-streaming GEMM launched next can start reading its weights while they run (see
    linear.nvfp4_linear).

    Returns:
        (packed, sf_swizzled, global_scale, alpha): alpha is None without gs_other.
    """
    if x.device.type != "cuda":
        raise ValueError("quantize_nvfp4_act needs a CUDA tensor")
    rows, k = x.shape
    if k % SF_VEC:
        raise ValueError("K must be a multiple of 16")
    dev = x.device
    src = (x if x.dtype in _IN_DTYPES else x.float()).contiguous()
    packed = torch.empty(rows, k // 2, dtype=torch.uint8, device=dev)
    sf_swz = torch.empty(sf_swizzled_size(rows, k), dtype=torch.uint8, device=dev)
    gs = torch.empty(1, dtype=torch.float32, device=dev)
    ws = torch.empty(_lib.ACT_WORKSPACE_BYTES // 4, dtype=torch.int32, device=dev)
    alpha = None
    other = None
    if gs_other is not None:
        other = gs_other.reshape(1).to(device=dev, dtype=torch.float32)
        alpha = torch.empty(1, dtype=torch.float32, device=dev)
    with torch.cuda.device(dev):
        rc = _lib.lib().nvfp4_quantize_act(
            src.data_ptr(), _IN_DTYPES[src.dtype], rows, k, other.data_ptr() if other is not None else None,
            gs.data_ptr(), alpha.data_ptr() if alpha is not None else None, packed.data_ptr(), sf_swz.data_ptr(),
            ws.data_ptr(), _stream(dev),
        )
    _lib.check(rc, "nvfp4_quantize_act")
    return packed, sf_swz, gs, alpha
