"""CPU: pin the C oracle against golden vectors produced by the reference package itself
(tests/golden/make_golden.py) and against PyTorch's float8_e4m3fn cast."""

import numpy as np
import pytest
import torch

from oracle import oracle
from tests.conftest import golden_cases


def _x(golden, name):
    return golden[f"{name}/x"]


def test_golden_cases_present(golden):
    assert set(golden_cases(golden)) >= {"ties", "randn_bf16", "randn_gs_f32", "outliers_bf16", "small_f16",
                                          "overflow"}


@pytest.mark.parametrize("name", ["ties", "randn_bf16", "randn_gs_f32", "outliers_bf16", "small_f16", "overflow"])
def test_quantize_matches_reference(golden, name):
    gs = float(golden[f"{name}/gs"][0])
    packed, sf_swz, sf_lin = oracle.quantize(_x(golden, name), gs, div_mode=1)
    np.testing.assert_array_equal(packed, golden[f"{name}/packed"])
    np.testing.assert_array_equal(sf_lin, golden[f"{name}/sf_linear"])
    np.testing.assert_array_equal(sf_swz, golden[f"{name}/sf_swizzled"])


@pytest.mark.parametrize("name", ["ties", "randn_gs_f32", "small_f16", "overflow"])
def test_dequantize_matches_reference(golden, name):
    gs = float(golden[f"{name}/gs"][0])
    out = oracle.dequantize(golden[f"{name}/packed"], golden[f"{name}/sf_linear"], gs, div_mode=1)
    assert_same_floats(out, golden[f"{name}/dequant"])


def assert_same_floats(got, want):
    """Bit-identical where finite or infinite (signed zeros included); NaN where the reference
    has NaN (NaN payloads are not part of the contract: CUDA arithmetic canonicalises them)."""
    got_nan, want_nan = np.isnan(got), np.isnan(want)
    np.testing.assert_array_equal(got_nan, want_nan)
    np.testing.assert_array_equal(got.view(np.uint32)[~want_nan], want.view(np.uint32)[~want_nan])


def test_swizzle_matches_reference(golden):
    np.testing.assert_array_equal(oracle.swizzle(golden["swizzle/in"]), golden["swizzle/out"])


def test_gemm_reference_fp32(golden):
    c = oracle.reference_fp32(golden["gemm/a_packed"], golden["gemm/a_sf_linear"], golden["gemm/b_packed"],
                              golden["gemm/b_sf_linear"])
    ref = golden["gemm/c_fp32"]
    # same FP32 products, different summation order between BLAS implementations
    assert np.linalg.norm(c - ref) / np.linalg.norm(ref) < 1e-6


def test_e4m3_matches_torch_cast():
    # every float32 bit pattern in the E4M3 range at a coarse stride, plus dense sweeps around
    # every rounding midpoint and the overflow boundary
    coarse = np.arange(0, 0x44000000, 97, dtype=np.uint32).view(np.float32)
    mids = []
    for b in range(0, 0x7F):
        lo = torch.tensor([b], dtype=torch.uint8).view(torch.float8_e4m3fn).float().item()
        hi = torch.tensor([b + 1], dtype=torch.uint8).view(torch.float8_e4m3fn).float().item() if b < 0x7E else 480.0
        mid = np.float32((lo + hi) / 2)
        base = mid.view(np.uint32)
        mids.append(np.arange(base - 3, base + 4, dtype=np.uint32).view(np.float32))
    vals = np.concatenate([coarse, *mids, np.array([448, 464, 464.00003, 480, 1e30, np.inf, -np.inf, np.nan],
                                                   dtype=np.float32)])
    vals = np.concatenate([vals, -vals])
    ref = torch.from_numpy(vals).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    got = oracle.e4m3_encode(vals)
    nan_ref = (ref & 0x7F) == 0x7F
    np.testing.assert_array_equal(nan_ref, (got & 0x7F) == 0x7F)
    np.testing.assert_array_equal(ref[~nan_ref], got[~nan_ref])


def test_e2m1_tie_table():
    # exact ties go to the even code; within ~1e-6 above a tie toward an odd code still even
    q = np.array([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 1.2500005, 1.2500015, -0.1, 0.1, -0.0, 7.0, -9.0],
                 dtype=np.float32)
    want = np.array([0, 2, 2, 4, 4, 6, 6, 2, 3, 8, 0, 0, 7, 15], dtype=np.uint8)
    np.testing.assert_array_equal(oracle.e2m1_code(q), want)


def test_div_modes_differ_only_where_torch_cpu_and_cuda_differ(golden):
    """Row 11 of the ties case has amax/6 one ulp below an E4M3 tie when divided exactly, and
    on the tie when multiplied by fl(1/6), as PyTorch does on CUDA. The golden vectors come from
    CPU tensors (exact division)."""
    x = _x(golden, "ties")
    _, _, sf_cpu = oracle.quantize(x, 1.0, div_mode=1)
    _, _, sf_cuda = oracle.quantize(x, 1.0, div_mode=0)
    np.testing.assert_array_equal(sf_cpu, golden["ties/sf_linear"])
    diff = np.nonzero(sf_cpu[:, 0] != sf_cuda[:, 0])[0].tolist()
    assert diff == [11]
    assert sf_cpu[11, 0] == 0x39 and sf_cuda[11, 0] == 0x3A  # 1.125 vs 1.25


def test_oracle_is_multithreaded():
    assert oracle.num_threads() >= 1
