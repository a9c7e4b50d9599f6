"""GPU: elementwise parity of the GEMM on the persistent path and on every BASELINE workload.

Each CTA pair of the default kernel computes several 256x256 tiles in a row as soon as a GEMM has
more tiles than there are pairs (74 on a B200): the second and later tiles of a pair, the
accumulator hand-off between them and the raster order that maps a work index to a tile are
exercised here at 4096^3 and above, each output element compared with the FP64 product of the
dequantised operands (the reference's quantise + dequantised-matmul path, nvfp4_gemm_cute/
testing.py:18-27, with FP64 in place of FP32).

Inputs follow the benchmark recipe: seeded N(0, 1) BF16 quantised with the per-tensor global
scale 2688 / amax on the device, alpha = 1 / (gs_A * gs_B) (docs/usage.md:14 of the reference).

Bars, as the north star states them:
  * relative Frobenius error <= 1e-3 against the FP64 result (BF16 output: against the FP64
    result rounded to BF16, since BF16 rounding alone is ~1.7e-3);
  * >= 99.9 % of elements within 2 ulp of the output dtype.
Where a full FP64 product would be too large (32768^3), 128 rows x 128 columns spread over every
256-row and 256-column tile band are compared (as the reference's benchmarks/compare.py:189-197
samples), plus whole rows and whole columns through every tile they cross. cuBLASLt on the same
GPU is a second, independent implementation: the outputs must be bit-identical.
"""

import pytest
import torch

pytestmark = pytest.mark.gpu

FROB_BAR = 1e-3
ULP_BAR = 0.999


def _operand(rows, k, seed, std=1.0, outliers=0.0, boost_cols=0):
    """Seeded BF16 [rows, k] -> (packed, swizzled scales, linear scales, global scale) with the
    on-device global scale 2688 / amax. `outliers`: that fraction of entries (seeded positions)
    replaced by +-50 sigma; `boost_cols`: that many seeded columns scaled by 20."""
    import gemm3_b200 as g3

    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(rows, k, device="cuda", generator=g) * std
    if boost_cols:
        cols = torch.randperm(k, generator=torch.Generator().manual_seed(seed + 1))[:boost_cols].cuda()
        x[:, cols] *= 20.0
    x = x.to(torch.bfloat16)
    n_out = int(x.numel() * outliers)
    if n_out:
        pos = torch.randint(x.numel(), (n_out,), device="cuda", generator=g)
        sign = torch.randint(0, 2, (n_out,), device="cuda", generator=g).to(torch.bfloat16) * 2 - 1
        x.view(-1)[pos] = sign * (50.0 * std)
    q, sf, sfl, gs = g3.quantize_nvfp4_global(x)
    del x
    return q, sf, sfl, gs


def _deq64(q, sfl, rows=None):
    from gemm3_b200 import dequantize_nvfp4

    if rows is not None:
        q, sfl = q[rows], sfl[rows]
    return dequantize_nvfp4(q.contiguous(), sfl.contiguous()).double()


def _ulps(out, ref64):
    """|out - round(ref64)| in ulps of the output dtype (a monotone integer line over the bits)."""
    o = out.contiguous().view(torch.int16).to(torch.int32)
    r = ref64.to(out.dtype).contiguous().view(torch.int16).to(torch.int32)
    o = torch.where(o < 0, -(o & 0x7FFF), o)
    r = torch.where(r < 0, -(r & 0x7FFF), r)
    return (o - r).abs()


def _assert_close(out, ref64, what):
    diff = out.double() - (ref64 if out.dtype == torch.float16 else ref64.to(out.dtype).double())
    rel = (diff.norm() / ref64.norm()).item()
    within2 = (_ulps(out, ref64) <= 2).double().mean().item()
    assert torch.isfinite(out).all(), f"{what}: non-finite output"
    assert rel <= FROB_BAR and within2 >= ULP_BAR, f"{what}: rel_frob={rel:.3e} within2ulp={within2:.5f}"
    return rel, within2


def _band_samples(extent, tile=256, count=128, salt=0):
    """`count` indices covering every `tile`-wide band of [0, extent) (several per band when there
    are fewer bands), at offsets that move through the tile."""
    bands = -(-extent // tile)
    idx = []
    for i in range(count):
        b = i % bands
        off = (37 * i + 11 * salt + 5) % tile
        idx.append(min(b * tile + off, extent - 1))
    return torch.tensor(sorted(set(idx)), device="cuda")


def _full_check(out, a, b, alpha, what):
    aq, _, asfl, _ = a
    bq, _, bsfl, _ = b
    ref = float(alpha.item()) * (_deq64(aq, asfl) @ _deq64(bq, bsfl).T)
    res = _assert_close(out, ref, what)
    del ref
    torch.cuda.empty_cache()
    return res


def _sampled_check(out, a, b, alpha, what, n_rows=128, n_cols=128, full_lines=2):
    """Sampled rows x sampled columns over every tile band, plus `full_lines` whole rows and whole
    columns (every tile along them)."""
    aq, _, asfl, _ = a
    bq, _, bsfl, _ = b
    m, n = out.shape
    al = float(alpha.item())
    rows = _band_samples(m, count=n_rows, salt=1)
    cols = _band_samples(n, count=n_cols, salt=2)
    a_rows = _deq64(aq, asfl, rows)
    ref = al * (a_rows @ _deq64(bq, bsfl, cols).T)
    _assert_close(out[rows][:, cols], ref, f"{what} (sampled {len(rows)}x{len(cols)})")
    # whole rows: every column tile; B dequantised in slices to bound memory
    lines = rows[:: max(1, len(rows) // full_lines)][:full_lines]
    got = out[lines]
    ref_rows = torch.empty(len(lines), n, dtype=torch.float64, device="cuda")
    step = 4096
    for c0 in range(0, n, step):
        c1 = min(n, c0 + step)
        ref_rows[:, c0:c1] = al * (_deq64(aq, asfl, lines) @ _deq64(bq, bsfl, torch.arange(c0, c1, device="cuda")).T)
    _assert_close(got, ref_rows, f"{what} (whole rows)")
    clines = cols[:: max(1, len(cols) // full_lines)][:full_lines]
    got_c = out[:, clines].T.contiguous()
    ref_c = torch.empty(len(clines), m, dtype=torch.float64, device="cuda")
    b_c = _deq64(bq, bsfl, clines)
    for r0 in range(0, m, step):
        r1 = min(m, r0 + step)
        ref_c[:, r0:r1] = al * (b_c @ _deq64(aq, asfl, torch.arange(r0, r1, device="cuda")).T)
    _assert_close(got_c, ref_c, f"{what} (whole columns)")
    torch.cuda.empty_cache()


def _gemm(g3, a, b, dtype, config=None):
    alpha = (1.0 / (a[3] * b[3])).reshape(1).float()
    out = g3.gemm(a[0], b[0], a[1], b[1], alpha=alpha, out_dtype=dtype, config=config)
    return out, alpha


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_persistent_4096_vs_fp64_and_cublaslt(cuda_ext, dtype):
    """256 tiles over 74 CTA pairs: every pair computes 3-4 tiles in a row."""
    from gemm3_b200.cublaslt import gemm_cublaslt

    a = _operand(4096, 4096, seed=40)
    b = _operand(4096, 4096, seed=41)
    out, alpha = _gemm(cuda_ext, a, b, dtype)
    _full_check(out, a, b, alpha, f"4096^3 {dtype}")
    vendor = gemm_cublaslt(a[0], b[0], a[1], b[1], alpha=alpha, out_dtype=dtype)
    torch.cuda.synchronize()
    assert torch.equal(out, vendor), int((out != vendor).sum())
    assert cuda_ext.device_status() == 0


@pytest.mark.parametrize(
    "cfg_kwargs",
    [
        dict(cluster=(4, 2), fast_swz=2, raster_along_m=False),   # the 4096^3 preset's band
        dict(cluster=(8, 2), fast_swz=4, raster_along_m=False),
        dict(cluster=(2, 1), fallback=None, raster_along_m=True),  # bands of N tiles
        dict(tile=(128, 256), cluster=(1, 1)),                     # one-CTA kernel, 512 tiles
    ],
)
def test_raster_orders_vs_fp64(cuda_ext, cfg_kwargs):
    """Every tile lands where it belongs whatever the raster: a tile computed for one position
    and stored at another would fail the elementwise comparison (a row sum could not see it)."""
    from gemm3_b200 import Config

    a = _operand(4096, 4096, seed=42)
    b = _operand(3072, 4096, seed=43)
    out, alpha = _gemm(cuda_ext, a, b, torch.float16, Config.make(**cfg_kwargs))
    _full_check(out, a, b, alpha, f"4096x3072x4096 {cfg_kwargs}")
    assert cuda_ext.device_status() == 0


@pytest.mark.parametrize("m,n,k", [(4000, 4032, 4096), (3329, 6080, 2240), (8191, 576, 1024)])
def test_ragged_persistent_vs_fp64(cuda_ext, m, n, k):
    """Several tiles per pair with partial last tiles in M and N and a K tail."""
    a = _operand(m, k, seed=m)
    b = _operand(n, k, seed=n)
    out, alpha = _gemm(cuda_ext, a, b, torch.bfloat16)
    _full_check(out, a, b, alpha, f"{m}x{n}x{k}")
    assert cuda_ext.device_status() == 0


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_config1_8192_vs_fp64_and_cublaslt(cuda_ext, dtype):
    """BASELINE config 1 (8192^3, BF16 out, the benchmark's workload and preset), in full; FP16
    as well. cuBLASLt on the same inputs gives the same bits."""
    from gemm3_b200.cublaslt import gemm_cublaslt

    a = _operand(8192, 8192, seed=0)
    b = _operand(8192, 8192, seed=1)
    out, alpha = _gemm(cuda_ext, a, b, dtype)
    _full_check(out, a, b, alpha, f"8192^3 {dtype}")
    vendor = gemm_cublaslt(a[0], b[0], a[1], b[1], alpha=alpha, out_dtype=dtype)
    torch.cuda.synchronize()
    assert torch.equal(out, vendor), int((out != vendor).sum())
    assert cuda_ext.device_status() == 0


def test_config2_16384_fp16_vs_fp64(cuda_ext):
    """BASELINE config 2 (16384^3, FP16 out, its preset), in full."""
    a = _operand(16384, 16384, seed=0)
    b = _operand(16384, 16384, seed=1)
    out, alpha = _gemm(cuda_ext, a, b, torch.float16)
    _full_check(out, a, b, alpha, "16384^3 fp16")
    assert cuda_ext.device_status() == 0


def test_config3_outliers_16384_bf16_vs_fp64(cuda_ext):
    """BASELINE config 3's inputs (0.1 % of entries replaced by +-50 sigma) at 16384^3, BF16
    out, in full."""
    a = _operand(16384, 16384, seed=0, outliers=1e-3)
    b = _operand(16384, 16384, seed=1, outliers=1e-3)
    out, alpha = _gemm(cuda_ext, a, b, torch.bfloat16)
    _full_check(out, a, b, alpha, "16384^3 bf16 outliers")
    assert cuda_ext.device_status() == 0


def test_config3_per_rank_shape_sampled(cuda_ext):
    """Config 3's per-GPU GEMM on 8 GPUs: 32768 x 4096 x 32768 with outliers, BF16 out; sampled
    rows and columns over every tile band, whole rows and columns."""
    a = _operand(32768, 32768, seed=0, outliers=1e-3)
    b = _operand(4096, 32768, seed=1, outliers=1e-3)
    out, alpha = _gemm(cuda_ext, a, b, torch.bfloat16)
    _sampled_check(out, a, b, alpha, "32768x4096x32768 bf16 outliers")
    assert cuda_ext.device_status() == 0


def test_32768_preset_sampled(cuda_ext):
    """32768^3 BF16 with its preset: 16384 tiles, ~221 per CTA pair."""
    a = _operand(32768, 32768, seed=0)
    b = _operand(32768, 32768, seed=1)
    out, alpha = _gemm(cuda_ext, a, b, torch.bfloat16)
    _sampled_check(out, a, b, alpha, "32768^3 bf16")
    assert cuda_ext.device_status() == 0


@pytest.mark.parametrize("m", [16, 128, 1024, 8192])
def test_config4_llm_projection_vs_fp64_and_cublaslt(cuda_ext, m):
    """W [28672, 8192] ~ N(0, 0.02), x [M, 8192] ~ N(0, 1) with 1 % of the
    columns x20, BF16 out. The library's call (nvfp4_linear: activation quantised on the GPU in
    the call) and the reference-API path (quantize_nvfp4_global + gemm with the shape's preset)
    give the same bits, within the bars of the FP64 product, and equal to cuBLASLt."""
    import gemm3_b200 as g3
    from gemm3_b200.cublaslt import gemm_cublaslt

    n, k = 28672, 8192
    w = _operand(n, k, seed=3, std=0.02)
    gx = torch.Generator(device="cuda").manual_seed(4)
    x = torch.randn(m, k, device="cuda", generator=gx)
    cols = torch.randperm(k, generator=torch.Generator().manual_seed(5))[: k // 100].cuda()
    x[:, cols] *= 20.0
    x = x.to(torch.bfloat16)
    y = g3.nvfp4_linear(x, w[0], w[1], w[3], out_dtype=torch.bfloat16)
    xq = g3.quantize_nvfp4_global(x)
    out, alpha = _gemm(cuda_ext, xq, w, torch.bfloat16)
    torch.cuda.synchronize()
    assert torch.equal(y, out), int((y != out).sum())
    _full_check(out, xq, w, alpha, f"LLM projection M={m}")
    vendor = gemm_cublaslt(xq[0], w[0], xq[1], w[1], alpha=alpha, out_dtype=torch.bfloat16)
    torch.cuda.synchronize()
    assert torch.equal(out, vendor), int((out != vendor).sum())
    assert cuda_ext.device_status() == 0


def test_back_to_back_launches_with_pdl(cuda_ext):
    """Consecutive GEMMs on one stream, launched with programmatic dependent launch (the default
    enable_pdl=True) and without, inside a CUDA graph and eagerly: the second GEMM reads the
    first one's output as its A operand's source only after quantisation, and every launch's
    output equals a lone launch's."""
    a = _operand(4096, 4096, seed=50)
    b = _operand(4096, 4096, seed=51)
    alpha = (1.0 / (a[3] * b[3])).reshape(1).float()
    ref = cuda_ext.gemm(a[0], b[0], a[1], b[1], alpha=alpha, out_dtype=torch.bfloat16, enable_pdl=False)
    outs = [torch.empty_like(ref) for _ in range(6)]

    def chain(pdl):
        for o in outs:
            cuda_ext.gemm(a[0], b[0], a[1], b[1], alpha=alpha, out=o, out_dtype=torch.bfloat16, enable_pdl=pdl)

    for pdl in (True, False):
        for o in outs:
            o.zero_()
        chain(pdl)
        torch.cuda.synchronize()
        for o in outs:
            assert torch.equal(o, ref)
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr, stream=side):
            chain(True)
    torch.cuda.current_stream().wait_stream(side)
    for o in outs:
        o.zero_()
    for _ in range(3):
        gr.replay()
    torch.cuda.synchronize()
    for o in outs:
        assert torch.equal(o, ref)
    # a dependent launch that consumes the previous GEMM's output: C1 -> quantise -> GEMM
    c1 = cuda_ext.gemm(a[0], b[0], a[1], b[1], alpha=alpha, out_dtype=torch.bfloat16)
    q1 = cuda_ext.quantize_nvfp4_global(c1)
    c2 = cuda_ext.gemm(q1[0], b[0], q1[1], b[1], out_dtype=torch.float16)
    torch.cuda.synchronize()
    q1_ref = cuda_ext.quantize_nvfp4_global(ref)
    c2_ref = cuda_ext.gemm(q1_ref[0], b[0], q1_ref[1], b[1], out_dtype=torch.float16, enable_pdl=False)
    torch.cuda.synchronize()
    assert torch.equal(c2, c2_ref)
    del gr
    assert cuda_ext.device_status() == 0
