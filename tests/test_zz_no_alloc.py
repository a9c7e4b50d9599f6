"""nvfp4_quantize_global_noalloc through the C ABI.

Global-scale quantisation needs one device float between its two kernels (the tensor amax).
The ordinary path has the caller allocate it. This entry point is for callers that cannot
allocate: a plugin or custom-call hook handed only its input and output buffers, or code that
must not call cudaMalloc while a stream capture is open or the device must not synchronise. It
keeps that float, and per-block partial maxima, in a fixed array inside the library. Its outputs
must equal the allocating path's (quantize_nvfp4_global: nvfp4_amax into a caller buffer, then
nvfp4_quantize) bit for bit, the quantiser tolerance used throughout these tests.

This file is named to be collected last, so a run that stops at the first failure has run every
other test before it.
"""

import ctypes

import pytest

from gemm3_b200 import _lib, build


def _call(L, x, packed, sf_swz, sf_lin, gs_out, stream):
    dtypes = {"torch.float16": _lib.DTYPE_F16, "torch.bfloat16": _lib.DTYPE_BF16, "torch.float32": _lib.DTYPE_F32}
    rows, k = x.shape
    return L.nvfp4_quantize_global_noalloc(
        x.data_ptr(), dtypes[str(x.dtype)], rows, k, packed.data_ptr(), sf_swz.data_ptr(), sf_lin.data_ptr(),
        gs_out.data_ptr(), stream,
    )


def test_noalloc_rejects_inputs_beyond_the_scratch_limit():
    """Validation answers before any device access, so this runs without a GPU."""
    build.build()
    L = _lib.lib()
    p = ctypes.c_void_p(1 << 20)  # never dereferenced
    k = 1 << 16
    rows = _lib.NOALLOC_MAX_ELEMENTS // k + 1
    assert L.nvfp4_quantize_global_noalloc(p, 1, rows, k, p, p, None, None, None) == _lib.ERR_TOO_LARGE
    assert b"2^31" in L.nvfp4_strerror(_lib.ERR_TOO_LARGE)
    # K not a multiple of 16 is an invalid value, as for nvfp4_quantize.
    assert L.nvfp4_quantize_global_noalloc(p, 1, 4, 24, p, p, None, None, None) == _lib.ERR_INVALID_VALUE


@pytest.mark.gpu
def test_noalloc_matches_quantize_global_on_two_calls_in_a_row(cuda_ext):
    import torch

    from gemm3_b200.quant import quantize_nvfp4_global, sf_swizzled_size

    L = _lib.lib()
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(7)
    # The first call is larger (more per-block partials) and has the larger amax; the second must
    # not see anything the first left in the shared array. Ragged row counts leave a partly
    # filled last block in both.
    cases = [
        (torch.randn(1000, 4096, generator=g, device=dev) * 3.0).to(torch.bfloat16),
        torch.randn(300, 512, generator=g, device=dev, dtype=torch.float32),
    ]
    for x in cases:
        rows, k = x.shape
        ref_packed, ref_swz, ref_lin, ref_gs = quantize_nvfp4_global(x)
        packed = torch.full((rows, k // 2), 0xAB, dtype=torch.uint8, device=dev)
        sf_swz = torch.full((sf_swizzled_size(rows, k),), 0xAB, dtype=torch.uint8, device=dev)
        sf_lin = torch.full((rows, k // 16), 0xAB, dtype=torch.uint8, device=dev)
        gs_out = torch.full((1,), -1.0, dtype=torch.float32, device=dev)
        rc = _call(L, x, packed, sf_swz, sf_lin, gs_out, torch.cuda.current_stream(dev).cuda_stream)
        assert rc == _lib.OK, L.nvfp4_strerror(rc)
        torch.cuda.synchronize(dev)
        assert torch.equal(gs_out.view(torch.int32), ref_gs.view(torch.int32)), (gs_out, ref_gs)
        assert torch.equal(packed, ref_packed)
        assert torch.equal(sf_swz, ref_swz)
        assert torch.equal(sf_lin, ref_lin)
