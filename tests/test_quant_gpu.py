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


def _boundary_blocks():
    """16-element FP32 blocks whose first element 6*d pins the block scale to the E4M3 value d;
    the other 15 are dividends within 24 ulps of d times each E2M1 rounding midpoint (and of
    their negatives), for every E4M3 significand at several exponents, including subnormal
    scales; plus blocks of zeros, signed zeros and tiny values next to a large scale."""
    blocks = []
    for e in (-9, -7, -6, -3, 0, 4, 7, 8):
        for m in range(8):
            d = np.float32((1.0 + m / 8.0) * 2.0**e)
            if d > 448.0 or (e < -6 and m != 0):
                continue
            for mid in (0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0):
                base = int(np.float32(np.float32(mid) * d).view(np.uint32))
                vals = (np.arange(base - 24, base + 24, dtype=np.int64).astype(np.uint32)).view(np.float32)
                vals = np.concatenate([vals, -vals])
                for i in range(0, len(vals) - 14, 15):
                    blocks.append(np.concatenate([[6.0 * d], vals[i:i + 15]]).astype(np.float32))
    tiny = np.float32([0.0, -0.0, 1e-45, -1e-45, 1e-40, -1e-38, 2.0**-101, -(2.0**-100), 2.0**-99, -1e-30,
                       3e-39, -3e-39, 0.0, -0.0, 7.0e-44])
    for d in (np.float32(448.0), np.float32(1.0), np.float32(2.0**-9)):
        blocks.append(np.concatenate([[6.0 * d], tiny]).astype(np.float32))
    while len(blocks) % 4:
        blocks.append(np.zeros(16, np.float32))
    return np.stack(blocks).reshape(-1, 64)


def test_quantize_near_rounding_boundaries(cuda_ext):
    """Division shortcut and threshold codes against the oracle's IEEE division and argmin."""
    x = _boundary_blocks()
    packed, sf_swz, sf_lin = cuda_ext.quantize_nvfp4(torch.from_numpy(x).cuda(), 1.0)
    want = oracle.quantize(x, 1.0, div_mode=0)
    np.testing.assert_array_equal(sf_lin.cpu().numpy(), want[2])
    np.testing.assert_array_equal(packed.cpu().numpy(), want[0])
    np.testing.assert_array_equal(sf_swz.cpu().numpy(), want[1])


def test_scale_encoding_sweep(cuda_ext):
    """Block scales at, and one ulp either side of, every E4M3 rounding midpoint (including 464,
    above which the reference's scale is NaN) and at every E4M3 value, through both roundings of
    '/ 6': the exact division (CPU tensors) and the multiply by fl(1/6) (CUDA tensors)."""
    vals = torch.arange(0x7F, dtype=torch.uint8).view(torch.float8_e4m3fn).float().numpy()
    vals = np.concatenate([vals, [480.0]]).astype(np.float32)  # 480: one step past 448
    s = []
    for a, b in zip(vals[:-1], vals[1:]):
        m = np.float32((np.float64(a) + np.float64(b)) / 2)
        s += [np.nextafter(m, np.float32(0)), m, np.nextafter(m, np.float32(1e9)), a]
    s = np.array(s, np.float32)
    amax = (s.astype(np.float64) * 6).astype(np.float32)  # exactly 6 m for the midpoints
    blocks = np.tile((amax * np.float32(0.5))[:, None], (1, 16)).astype(np.float32)
    blocks[:, 0] = amax
    blocks = np.concatenate([blocks, np.zeros(((-len(blocks)) % 4, 16), np.float32)])
    x = blocks.reshape(-1, 64)
    for xt, div_mode in ((torch.from_numpy(x), 1), (torch.from_numpy(x).cuda(), 0)):
        packed, sf_swz, sf_lin = cuda_ext.quantize_nvfp4(xt, 1.0)
        want = oracle.quantize(x, 1.0, div_mode=div_mode)
        np.testing.assert_array_equal(sf_lin.cpu().numpy(), want[2])
        np.testing.assert_array_equal(sf_swz.cpu().numpy(), want[1])
        np.testing.assert_array_equal(packed.cpu().numpy(), want[0])


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_quantize_output_alignment_paths_agree(cuda_ext, dtype):
    """16-bit inputs with k % 32 == 0 go to the two-blocks-per-thread kernel when the codes are
    16-byte and the scale arrays 2-byte aligned, else to the one-block kernel. Outputs written at
    odd offsets (through the C ABI) must hold the same bytes as aligned ones."""
    from gemm3_b200 import _lib
    from gemm3_b200.quant import sf_swizzled_size

    L = _lib.lib()
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(5)
    rows, k = 300, 2048
    x = (torch.randn(rows, k, device=dev, generator=g) * 4.0).to(dtype)
    code = _lib.DTYPE_BF16 if dtype == torch.bfloat16 else _lib.DTYPE_F16
    stream = torch.cuda.current_stream(dev).cuda_stream
    nsw = sf_swizzled_size(rows, k)
    outs = []
    for off_p, off_s in ((0, 0), (8, 1)):  # aligned; codes 8-byte and scales 1-byte aligned only
        packed = torch.zeros(rows * k // 2 + 16, dtype=torch.uint8, device=dev)
        sf_swz = torch.zeros(nsw + 2, dtype=torch.uint8, device=dev)
        sf_lin = torch.zeros(rows * k // 16 + 2, dtype=torch.uint8, device=dev)
        rc = L.nvfp4_quantize(x.data_ptr(), code, rows, k, 1.7, None, 0, 0, packed.data_ptr() + off_p,
                              sf_swz.data_ptr() + off_s, sf_lin.data_ptr() + off_s, None, stream)
        assert rc == _lib.OK, L.nvfp4_strerror(rc)
        outs.append((packed[off_p:off_p + rows * k // 2], sf_swz[off_s:off_s + nsw], sf_lin[off_s:off_s + rows * k // 16]))
    torch.cuda.synchronize()
    for a, b in zip(*outs):
        assert torch.equal(a, b)
    want = oracle.quantize(x.float().cpu().numpy(), 1.7, div_mode=0)
    np.testing.assert_array_equal(outs[0][0].cpu().numpy().reshape(rows, k // 2), want[0])
    np.testing.assert_array_equal(outs[0][1].cpu().numpy(), want[1])


def test_quantize_2pow32_elements_matches_row_slices(cuda_ext):
    """2^32 elements (8 GiB of BF16): the kernel walks the grid with 64-bit indices there, and
    with 32-bit ones for anything smaller. Row blocks at both ends (the last ones past 2^31 and
    near 2^32 elements) quantised on their own must give the same bytes, in all three outputs."""
    rows, k = 1 << 18, 1 << 14
    x = torch.empty(rows, k, device="cuda", dtype=torch.bfloat16)
    g = torch.Generator(device="cuda").manual_seed(11)
    for r0 in range(0, rows, 16384):
        x[r0:r0 + 16384] = torch.randn(16384, k, device="cuda", generator=g).to(torch.bfloat16)
    gs = torch.tensor([2688.0 / 5.5], device="cuda")
    packed, sf_swz, sf_lin = cuda_ext.quantize_nvfp4(x, gs)
    chunk = 128 * (k // 64) * 4  # swizzled scale bytes of one 128-row block
    for r0 in (0, (1 << 17) + 128, rows - 256):
        p2, s2, l2 = cuda_ext.quantize_nvfp4(x[r0:r0 + 256], gs)
        assert torch.equal(packed[r0:r0 + 256], p2)
        assert torch.equal(sf_lin[r0:r0 + 256], l2)
        assert torch.equal(sf_swz[r0 // 128 * chunk:(r0 // 128 + 2) * chunk], s2)
    del x, packed, sf_swz, sf_lin
    torch.cuda.empty_cache()


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
def test_amax_odd_sizes_and_nan(cuda_ext, dtype):
    # sizes around the kernel's 16-byte vectors (4 or 8 elements) and its four-load unroll
    for n in (1, 3, 7, 9, 15, 16, 17, 4095, 1000003):
        x = torch.randn(n, device="cuda").to(dtype)
        x[n // 2] = -7.5  # a negative maximum magnitude, anywhere in the vector stream
        assert cuda_ext.tensor_amax(x).item() == x.float().abs().max().item()
    for pos in (0, 123, 999):  # NaN in the vector body and in the tail
        x = torch.randn(1003, device="cuda").to(dtype)
        x[pos] = float("nan")
        assert torch.isnan(cuda_ext.tensor_amax(x)).item()
    x = torch.randn(1003, device="cuda").to(dtype)
    x[5] = float("-inf")
    assert cuda_ext.tensor_amax(x).item() == float("inf")


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


def _special_16bit_rows(dtype):
    """Rows of 16-bit inputs made of the values whose widening to FP32 needs care: signed zeros,
    subnormals of the input type, the largest finite values, infinities and NaN, each alone in a
    block and mixed with ordinary values."""
    fin = torch.finfo(dtype)
    sub = fin.tiny / 4  # a subnormal of the input type
    rng = np.random.default_rng(17)
    ordinary = rng.normal(size=16).astype(np.float32)
    rows = [
        [-0.0] * 16,
        [0.0, -0.0] * 8,
        [sub, -sub] * 8,
        [sub] + [0.0] * 15,
        [-sub, 1.0] + [-0.0] * 14,
        [fin.max, -fin.max] + list(ordinary[:14]),
        [float("inf")] + list(ordinary[:15]),
        [float("-inf"), -0.0] + list(ordinary[:14]),
        [float("nan")] + list(ordinary[:15]),
        list(ordinary[:8]) + [-0.0, 0.0, sub, -sub, fin.tiny, -fin.tiny, 1.0, -1.0],
        list(ordinary),
        list(-ordinary),
    ]
    x = torch.tensor(rows, dtype=torch.float32).to(dtype)
    return torch.cat([x, x.flip(1)], dim=1)  # 12 rows x 32 elements: both pair-kernel block slots


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("gs", [1.0, 448.0, 3.0e-3])
def test_quantize_16bit_special_values_match_oracle(cuda_ext, dtype, gs):
    """Signed zeros, subnormals, the largest finite values, infinities and NaN of 16-bit inputs,
    through the two-block kernel (k % 32 == 0) and the one-block kernel (k = 48), bit for bit
    against the oracle on the same values widened to FP32."""
    x = _special_16bit_rows(dtype)
    for xk in (x, torch.cat([x, x[:, :16]], dim=1)):
        packed, sf_swz, sf_lin = cuda_ext.quantize_nvfp4(xk.cuda(), gs)
        want = oracle.quantize(xk.float().numpy(), gs, div_mode=0)
        np.testing.assert_array_equal(packed.cpu().numpy(), want[0])
        np.testing.assert_array_equal(sf_lin.cpu().numpy(), want[2])
        np.testing.assert_array_equal(sf_swz.cpu().numpy(), want[1])
