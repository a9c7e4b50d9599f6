"""GPU: the CUDA quantiser, dequantiser, swizzle and amax against the golden vectors and the
oracle, bit for bit."""

import numpy as np
import pytest
import torch

from oracle import oracle
from tests.conftest import golden_cases
from tests.test_oracle_golden import assert_same_floats

pytestmark = pytest.mark.gpu

_TORCH_DTYPES = {"float32": torch.float32, "bfloat16": torch.bfloat16, "float16": torch.float16}


def _input(golden, name):
    x = torch.from_numpy(golden[f"{name}/x"])
    return x.to(_TORCH_DTYPES[str(golden[f"{name}/dtype"])])


@pytest.mark.parametrize("name", ["ties", "randn_bf16", "randn_gs_f32", "outliers_bf16", "small_f16", "overflow"])
def test_quantize_cpu_tensor_matches_reference_golden(cuda_ext, golden, name):
    """CPU tensors in, like the golden run: the kernel uses the CPU rounding of '/ 6'."""
    gs = float(golden[f"{name}/gs"][0])
    packed, sf_swz, sf_lin = cuda_ext.quantize_nvfp4(_input(golden, name), gs)
    assert packed.device.type == "cpu"
    np.testing.assert_array_equal(packed.numpy(), golden[f"{name}/packed"])
    np.testing.assert_array_equal(sf_lin.numpy(), golden[f"{name}/sf_linear"])
    np.testing.assert_array_equal(sf_swz.numpy(), golden[f"{name}/sf_swizzled"])


@pytest.mark.parametrize("name", ["ties", "randn_bf16", "randn_gs_f32", "outliers_bf16", "small_f16", "overflow"])
def test_quantize_cuda_tensor_matches_oracle(cuda_ext, golden, name):
    gs = float(golden[f"{name}/gs"][0])
    x = _input(golden, name)
    packed, sf_swz, sf_lin = cuda_ext.quantize_nvfp4(x.cuda(), gs)
    want = oracle.quantize(golden[f"{name}/x"], gs, div_mode=0)
    np.testing.assert_array_equal(packed.cpu().numpy(), want[0])
    np.testing.assert_array_equal(sf_swz.cpu().numpy(), want[1])
    np.testing.assert_array_equal(sf_lin.cpu().numpy(), want[2])


def test_cuda_scalar_division_is_reciprocal_multiply(cuda_ext):
    """Pins the assumption behind div_mode 0: PyTorch on CUDA computes t / 6.0 as t * fl(1/6),
    which rounds differently from the exact division on one crafted value."""
    t = torch.tensor([7.125 - 2.0**-21], dtype=torch.float32)
    on_cuda = (t.cuda() / 6.0).to(torch.float8_e4m3fn).view(torch.uint8).item()
    on_cpu = (t / 6.0).to(torch.float8_e4m3fn).view(torch.uint8).item()
    assert on_cpu == oracle.e4m3_encode(np.array([np.float32(t.item()) / np.float32(6.0)]))[0] == 0x39
    assert on_cuda == 0x3A


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("shape", [(4096, 4096), (1000, 8192), (1, 64), (129, 48)])
def test_quantize_random_large(cuda_ext, dtype, shape):
    g = torch.Generator(device="cuda").manual_seed(7)
    x = torch.randn(*shape, device="cuda", generator=g)
    x.view(-1)[:: 997] *= 50.0  # outliers
    x = x.to(dtype)
    amax = x.float().abs().max()
    gs = float(torch.tensor(2688.0, device="cuda") / amax)
    packed, sf_swz, sf_lin = cuda_ext.quantize_nvfp4(x, gs)
    want = oracle.quantize(x.float().cpu().numpy(), gs, div_mode=0)
    np.testing.assert_array_equal(packed.cpu().numpy(), want[0])
    np.testing.assert_array_equal(sf_lin.cpu().numpy(), want[2])
    np.testing.assert_array_equal(sf_swz.cpu().numpy(), want[1])


def test_quantize_global_scale_on_device(cuda_ext):
    g = torch.Generator(device="cuda").manual_seed(3)
    x = (torch.randn(512, 2048, device="cuda", generator=g) * 3).to(torch.bfloat16)
    packed, sf_swz, sf_lin, gs = cuda_ext.quantize_nvfp4_global(x)
    amax = x.float().abs().max()
    gs_ref = torch.tensor(2688.0, device="cuda") / amax
    assert gs.item() == gs_ref.item()
    assert cuda_ext.tensor_amax(x).item() == amax.item()
    want = oracle.quantize(x.float().cpu().numpy(), gs_ref.item(), div_mode=0)
    np.testing.assert_array_equal(packed.cpu().numpy(), want[0])
    np.testing.assert_array_equal(sf_swz.cpu().numpy(), want[1])
    # a device tensor as global_scale gives the same result
    p2, s2, _ = cuda_ext.quantize_nvfp4(x, gs)
    assert torch.equal(p2, packed) and torch.equal(s2, sf_swz)


def test_amax_odd_sizes_and_nan(cuda_ext):
    for n in (1, 15, 16, 17, 1000003):
        x = torch.randn(n, device="cuda")
        assert cuda_ext.tensor_amax(x).item() == x.abs().max().item()
    x = torch.randn(1000, device="cuda")
    x[123] = float("nan")
    assert torch.isnan(cuda_ext.tensor_amax(x)).item()


@pytest.mark.parametrize("name", ["ties", "randn_gs_f32", "small_f16", "overflow"])
def test_dequantize_matches_reference_golden(cuda_ext, golden, name):
    gs = float(golden[f"{name}/gs"][0])
    packed = torch.from_numpy(golden[f"{name}/packed"])
    sfl = torch.from_numpy(golden[f"{name}/sf_linear"])
    out_cpu = cuda_ext.dequantize_nvfp4(packed, sfl, gs)  # CPU tensors: exact division by gs
    assert_same_floats(out_cpu.numpy(), golden[f"{name}/dequant"])
    out_gpu = cuda_ext.dequantize_nvfp4(packed.cuda(), sfl.cuda(), gs)  # CUDA: multiply by fl(1/gs)
    assert_same_floats(out_gpu.cpu().numpy(), oracle.dequantize(packed.numpy(), sfl.numpy(), gs, div_mode=0))


def test_swizzle_matches_reference_golden(cuda_ext, golden):
    sf = torch.from_numpy(golden["swizzle/in"])
    np.testing.assert_array_equal(cuda_ext.swizzle_sf(sf.cuda()).cpu().numpy(), golden["swizzle/out"])


def test_no_device_errors(cuda_ext):
    assert cuda_ext.device_status() == 0
