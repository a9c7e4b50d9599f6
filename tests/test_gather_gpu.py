"""GPU: the output view of nvfp4_gemm_run_gather on one GPU (destination list of one buffer).

Each kernel (CTA pair, one CTA, weight-streaming) writes its [M, N] block at columns
[col0, col0 + N) of a wider row-major [M, ldc] buffer, bit-identical to gemm() into a contiguous
output, and leaves every other column untouched. The peer destinations of the same entry point
are covered by tests/test_dist_gpu.py on two GPUs.
"""

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("tile,m", [((256, 256), 300), ((128, 256), 200), ((128, 128), 64), ((128, 128), 5)])
def test_gather_view_single_destination(cuda_ext, tile, m):
    from gemm3_b200 import Config, _lib
    from gemm3_b200.api import _launch_config
    from gemm3_b200.testing import make_inputs

    n, k, col0, ldc = 576, 1088, 64, 832
    inp = make_inputs(m, n, k, seed=m + tile[1])
    cfg = Config.make(tile=tile)
    alpha = torch.tensor([0.75], device="cuda")
    want = cuda_ext.gemm(inp["a"], inp["b"], inp["a_sf"], inp["b_sf"], alpha=alpha, out_dtype=torch.bfloat16,
                         config=cfg)
    buf = torch.full((m, ldc), -7.0, dtype=torch.bfloat16, device="cuda")
    dst = (ctypes.c_void_p * 1)(buf.data_ptr())
    ccfg = _launch_config(m, k, cfg, {}, 0)
    rc = _lib.lib().nvfp4_gemm_run_gather(
        inp["a"].data_ptr(), inp["b"].data_ptr(), inp["a_sf"].data_ptr(), inp["b_sf"].data_ptr(), dst, 1, ldc, col0,
        alpha.data_ptr(), m, n, k, _lib.DTYPE_BF16, ctypes.byref(ccfg), None, torch.cuda.current_stream().cuda_stream,
    )
    assert rc == _lib.OK
    torch.cuda.synchronize()
    assert torch.equal(buf[:, col0 : col0 + n], want)
    assert bool((buf[:, :col0] == -7.0).all()) and bool((buf[:, col0 + n :] == -7.0).all())
