"""GPU: the tcgen05 GEMM against cuBLASLt's NVFP4 GEMM on the same B200, bit for bit.

cuBLASLt (libgemm3_b200_cublaslt.so) is a second, independent implementation of the same block-
scaled product. The reference records every library it benchmarks as bit-identical to its own
kernel (benchmarks/results/libraries-*.json); the same holds here for both output dtypes, ragged
and skinny M and K tails.
"""

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("m,n,k", [(256, 256, 256), (1000, 1024, 768), (129, 320, 1088), (16, 2048, 4096),
                                   (2048, 2048, 2048)])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_bit_identical_to_cublaslt(cuda_ext, m, n, k, dtype):
    from gemm3_b200.cublaslt import gemm_cublaslt
    from gemm3_b200.testing import make_inputs

    inp = make_inputs(m, n, k, seed=m + n + k)
    alpha = torch.tensor([0.8125], device="cuda")
    ours = cuda_ext.gemm(inp["a"], inp["b"], inp["a_sf"], inp["b_sf"], alpha=alpha, out_dtype=dtype)
    vendor = gemm_cublaslt(inp["a"], inp["b"], inp["a_sf"], inp["b_sf"], alpha=0.8125, out_dtype=dtype)
    torch.cuda.synchronize()
    assert torch.equal(ours, vendor), int((ours != vendor).sum())
