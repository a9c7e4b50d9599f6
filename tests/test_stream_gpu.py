"""GPU: the weight-streaming kernel (tile (128, 128), the M <= 128 preset).

It computes C^T = B . A^T with B's rows in the tensor core's M dimension and all of A's rows in
its N. Each output element is still one MMA chain over k = 0, 64, 128, ..., so the result is
checked bit for bit against the one-CTA 128x256 kernel, besides the FP64 oracle. Ragged N (a
64-row last tile), K tails (1-7 scale blocks in the last 512-element stage), every A-row count
class (1, 8, 16 ... 128 rows; MMA N of 16-128), both output dtypes, alpha, and the programmatic
dependent launch modes, including inside a CUDA graph.
"""

import ctypes

import pytest
import torch

from oracle import oracle

pytestmark = pytest.mark.gpu

ONE_CTA = dict(tile=(128, 256))
STREAM = dict(tile=(128, 128))


def _inputs(m, n, k, seed):
    from gemm3_b200.testing import make_inputs

    return make_inputs(m, n, k, seed=seed)


def _rel_and_within2(out, c64):
    ref = torch.from_numpy(c64).cuda()
    rel = ((out.double() - ref).norm() / ref.norm()).item()
    o = out.view(torch.int16).to(torch.int32)
    r = ref.to(out.dtype).view(torch.int16).to(torch.int32)
    o = torch.where(o < 0, -(o & 0x7FFF), o)
    r = torch.where(r < 0, -(r & 0x7FFF), r)
    return rel, ((o - r).abs() <= 2).double().mean().item()


@pytest.mark.parametrize(
    "m,n,k",
    [(1, 64, 64), (8, 512, 1024), (16, 1024, 2048), (24, 768, 576), (33, 192, 1088), (64, 320, 4096),
     (100, 1088, 704), (128, 256, 512), (128, 2048, 8192)],
)
def test_stream_vs_oracle_and_one_cta_bits(cuda_ext, m, n, k):
    from gemm3_b200 import Config

    inp = _inputs(m, n, k, seed=m * 7 + n + k)
    args = (inp["a"], inp["b"], inp["a_sf"], inp["b_sf"])
    out = cuda_ext.gemm(*args, config=Config.make(**STREAM))
    c64 = oracle.gemm_fp64(*(inp[x].cpu().numpy() for x in ("a", "a_sf_linear", "b", "b_sf_linear")))
    rel, within2 = _rel_and_within2(out, c64)
    assert rel <= 1e-3 and within2 >= 0.999, (rel, within2)
    base = cuda_ext.gemm(*args, config=Config.make(**ONE_CTA))
    assert torch.equal(out, base), int((out != base).sum())
    assert cuda_ext.device_status() == 0


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_stream_alpha_and_dtype(cuda_ext, dtype):
    from gemm3_b200 import Config

    inp = _inputs(48, 640, 1536, seed=11)
    args = (inp["a"], inp["b"], inp["a_sf"], inp["b_sf"])
    alpha = torch.tensor([0.3125], device="cuda")
    out = cuda_ext.gemm(*args, alpha=alpha, out_dtype=dtype, config=Config.make(**STREAM))
    base = cuda_ext.gemm(*args, alpha=alpha, out_dtype=dtype, config=Config.make(**ONE_CTA))
    assert torch.equal(out, base)


def test_stream_is_the_skinny_preset(cuda_ext):
    """config_for picks the stream kernel for M <= 128; the default call equals the explicit one."""
    from gemm3_b200 import Config, config_for

    assert config_for(16, 28672, 8192).tile == (128, 128)
    inp = _inputs(16, 28672 // 8, 8192, seed=3)
    args = (inp["a"], inp["b"], inp["a_sf"], inp["b_sf"])
    assert torch.equal(cuda_ext.gemm(*args), cuda_ext.gemm(*args, config=Config.make(**STREAM)))


def _c_launch(L, inp, out, alpha, pdl, stream):
    from gemm3_b200 import _lib

    cfg = _lib.GemmConfig()
    cfg.struct_size = ctypes.sizeof(cfg)
    cfg.tile_m, cfg.tile_n, cfg.pdl = 128, 128, pdl
    m, n, k = inp["a"].shape[0], inp["b"].shape[0], inp["a"].shape[1] * 2
    return L.nvfp4_gemm_run(
        inp["a"].data_ptr(), inp["b"].data_ptr(), inp["a_sf"].data_ptr(), inp["b_sf"].data_ptr(), out.data_ptr(),
        alpha.data_ptr(), m, n, k, _lib.DTYPE_BF16, ctypes.byref(cfg), None, stream,
    )


def test_stream_pdl_modes_through_c_abi_and_graph(cuda_ext):
    """pdl 0, 1 and 2 give the same bits; mode 2 follows the kernel that quantises A (and writes
    alpha) in the same stream, eagerly and inside a captured CUDA graph."""
    from gemm3_b200 import _lib, quantize_nvfp4_global

    L = _lib.lib()
    torch.manual_seed(0)
    x = torch.randn(16, 4096, device="cuda").to(torch.bfloat16)
    w = (torch.randn(1536, 4096, device="cuda") * 0.02).to(torch.bfloat16)
    wq, wsf, _, gs_w = quantize_nvfp4_global(w)
    outs = []
    stream = torch.cuda.current_stream().cuda_stream
    for pdl in (0, 1, 2):
        xq, xsf, _, gs_x = quantize_nvfp4_global(x)
        alpha = torch.reciprocal(gs_x * gs_w)
        out = torch.empty(16, 1536, dtype=torch.bfloat16, device="cuda")
        inp = {"a": xq, "b": wq, "a_sf": xsf, "b_sf": wsf}
        assert _c_launch(L, inp, out, alpha, pdl, stream) == _lib.OK
        outs.append(out)
    torch.cuda.synchronize()
    assert torch.equal(outs[0], outs[1]) and torch.equal(outs[0], outs[2])

    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    out_g = torch.empty(16, 1536, dtype=torch.bfloat16, device="cuda")
    with torch.cuda.stream(s):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            xq2, xsf2, _, gs_x2 = quantize_nvfp4_global(x)
            alpha2 = torch.reciprocal(gs_x2 * gs_w)
            inp = {"a": xq2, "b": wq, "a_sf": xsf2, "b_sf": wsf}
            assert _c_launch(L, inp, out_g, alpha2, 2, s.cuda_stream) == _lib.OK
    torch.cuda.current_stream().wait_stream(s)
    for _ in range(3):
        out_g.zero_()
        g.replay()
        torch.cuda.synchronize()
        assert torch.equal(out_g, outs[0])
    del g
    assert cuda_ext.device_status() == 0


@pytest.mark.parametrize(
    "rows,k,dtype",
    [(1, 64, torch.bfloat16), (16, 8192, torch.bfloat16), (100, 1040, torch.float16), (128, 8192, torch.float32),
     (300, 4096, torch.bfloat16), (2048, 8192, torch.bfloat16)],
)
def test_quantize_act_equals_global(cuda_ext, rows, k, dtype):
    """The activation quantiser (amax partials + quantiser, chained by programmatic dependent
    launch) == quantize_nvfp4_global, bit for bit; alpha == torch's reciprocal(gs_x * gs_w)."""
    from gemm3_b200 import quantize_nvfp4_act, quantize_nvfp4_global

    g = torch.Generator(device="cuda").manual_seed(rows + k)
    x = torch.randn(rows, k, device="cuda", generator=g)
    x[:, ::97] *= 20.0
    x = x.to(dtype)
    gs_w = torch.tensor([1234.5], device="cuda")
    q, sf, gs, alpha = quantize_nvfp4_act(x, gs_w)
    q0, sf0, _, gs0 = quantize_nvfp4_global(x)
    torch.cuda.synchronize()
    assert torch.equal(gs.view(torch.int32), gs0.view(torch.int32))
    assert torch.equal(q, q0) and torch.equal(sf, sf0)
    assert torch.equal(alpha.view(torch.int32), torch.reciprocal(gs0 * gs_w).view(torch.int32))


@pytest.mark.parametrize("fill", [0.0, float("inf"), float("nan")])
def test_quantize_act_degenerate_amax(cuda_ext, fill):
    """amax 0, Inf or NaN: gs = 1, as quantize_nvfp4_global."""
    from gemm3_b200 import quantize_nvfp4_act, quantize_nvfp4_global

    x = torch.zeros(8, 256, device="cuda", dtype=torch.bfloat16)
    x[3, 17] = fill
    x[5, 0] = 0.5
    if fill == 0.0:
        x.zero_()
    q, sf, gs, _ = quantize_nvfp4_act(x)
    q0, sf0, _, gs0 = quantize_nvfp4_global(x)
    torch.cuda.synchronize()
    assert gs.item() == 1.0 and torch.equal(gs.view(torch.int32), gs0.view(torch.int32))
    assert torch.equal(q, q0) and torch.equal(sf, sf0)


@pytest.mark.parametrize("m", [1, 16, 128, 129])
def test_nvfp4_linear_equals_quantise_then_gemm(cuda_ext, m):
    """The LLM-projection call (activation quantiser, then the GEMM overlapping it) == the
    three-step path of the reference's API, bit for bit, eagerly and replayed from a graph."""
    from gemm3_b200 import gemm, nvfp4_linear, quantize_nvfp4_global

    g = torch.Generator(device="cuda").manual_seed(m)
    w = (torch.randn(2304, 2048, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    wq, wsf, _, gs_w = quantize_nvfp4_global(w)
    x = torch.randn(m, 2048, device="cuda", generator=g).to(torch.bfloat16)
    xq, xsf, _, gs_x = quantize_nvfp4_global(x)
    ref = gemm(xq, wq, xsf, wsf, alpha=torch.reciprocal(gs_x * gs_w), out_dtype=torch.bfloat16)
    y = nvfp4_linear(x, wq, wsf, gs_w)
    torch.cuda.synchronize()
    assert torch.equal(y, ref)

    out = torch.empty_like(ref)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        nvfp4_linear(x, wq, wsf, gs_w, out=out)  # warm-up outside capture
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=s):
            nvfp4_linear(x, wq, wsf, gs_w, out=out)
    torch.cuda.current_stream().wait_stream(s)
    for _ in range(2):
        out.zero_()
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(out, ref)
    del graph
    assert cuda_ext.device_status() == 0
