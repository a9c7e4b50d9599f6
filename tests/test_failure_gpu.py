"""GPU: failure detection without a GPU fault.

A device-side wait that can never complete (an mbarrier nothing arrives at, through the bounded
wait every GEMM kernel uses) ends after its limit with a status word instead of a hang, and the
context stays usable: a GEMM launched afterwards still matches the oracle.
"""

import time

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_unfinishable_wait_reports_timeout_and_context_survives(cuda_ext):
    from gemm3_b200 import _lib
    from gemm3_b200.testing import make_inputs, reference

    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    t0 = time.monotonic()
    rc = _lib.lib().nvfp4_selftest_wait_timeout(status.data_ptr(), 103, torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    torch.cuda.synchronize()
    waited = time.monotonic() - t0
    assert status.item() == 103  # NVFP4_DEV_TIMEOUT_ACC_FULL, the code the test asked for
    assert 1.0 < waited < 30.0, waited  # the wait gave up after its ~2 s limit
    assert b"timeout" in _lib.lib().nvfp4_strerror(103)

    inp = make_inputs(256, 512, 512, seed=9)
    out = cuda_ext.gemm(inp["a"], inp["b"], inp["a_sf"], inp["b_sf"])
    ref = reference(inp)
    assert ((out.float() - ref).norm() / ref.norm()).item() < 2e-3
    assert cuda_ext.device_status() == 0
