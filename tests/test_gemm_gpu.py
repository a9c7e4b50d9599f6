"""GPU: the tcgen05 NVFP4 GEMM against the reference's FP32 check, the FP64 oracle and itself
across launch configurations (the reference's tests/test_gemm.py, re-targeted at sm_100)."""

import numpy as np
import pytest
import torch

from oracle import oracle

pytestmark = pytest.mark.gpu


def _inputs(cuda_ext, m, n, k, seed=0):
    from gemm3_b200.testing import make_inputs

    return make_inputs(m, n, k, seed=seed)


def _fp64_reference(inp, alpha=1.0):
    from gemm3_b200 import dequantize_nvfp4

    a = dequantize_nvfp4(inp["a"], inp["a_sf_linear"]).double()
    b = dequantize_nvfp4(inp["b"], inp["b_sf_linear"]).double()
    return alpha * (a @ b.T)


def _ulp_distance(out, ref64):
    """|out - round(ref64)| in units of the output dtype's ulp at round(ref64)."""
    ref_r = ref64.to(out.dtype)
    o = out.view(torch.int16).to(torch.int32)
    r = ref_r.view(torch.int16).to(torch.int32)
    # map sign-magnitude to a monotone integer line
    o = torch.where(o < 0, -(o & 0x7FFF), o)
    r = torch.where(r < 0, -(r & 0x7FFF), r)
    return (o - r).abs()


def _accuracy(out, ref64):
    rel = ((out.double() - ref64).norm() / ref64.norm()).item()
    rel_rounded = ((out.double() - ref64.to(out.dtype).double()).norm() / ref64.norm()).item()
    within2 = (_ulp_distance(out, ref64) <= 2).double().mean().item()
    return rel, rel_rounded, within2


@pytest.mark.parametrize("m,n,k", [(512, 512, 512), (1000, 1024, 768), (2048, 1536, 4096)])
def test_default_config(cuda_ext, m, n, k):
    from gemm3_b200.testing import check, reference

    inp = _inputs(cuda_ext, m, n, k)
    out = cuda_ext.gemm(inp["a"], inp["b"], inp["a_sf"], inp["b_sf"])
    ok, err = check(out, reference(inp))
    assert ok, err


def test_golden_gemm(cuda_ext, golden):
    """The reference's FP32 result for committed packed inputs (tests/golden/make_golden.py)."""
    t = {k.split("/")[1]: torch.from_numpy(v).cuda() for k, v in golden.items() if k.startswith("gemm/")}
    out = cuda_ext.gemm(t["a_packed"], t["b_packed"], t["a_sf"], t["b_sf"])
    ref = t["c_fp32"]
    err = ((out.float() - ref).norm() / ref.norm()).item()
    assert err < 2e-3, err
    c64 = oracle.gemm_fp64(golden["gemm/a_packed"], golden["gemm/a_sf_linear"], golden["gemm/b_packed"],
                           golden["gemm/b_sf_linear"])
    rel, _, within2 = _accuracy(out, torch.from_numpy(c64).cuda())
    assert rel <= 1e-3 and within2 >= 0.999, (rel, within2)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_accuracy_contract_fp64(cuda_ext, dtype):
    """rel. Frobenius <= 1e-3 against FP64 (FP16 out; BF16 rounding alone exceeds it, so BF16 is
    held to the same bound against the FP64 result rounded to BF16), and >= 99.9% of elements
    within 2 ulp of the output dtype."""
    inp = _inputs(cuda_ext, 2048, 2048, 2048, seed=5)
    out = cuda_ext.gemm(inp["a"], inp["b"], inp["a_sf"], inp["b_sf"], out_dtype=dtype)
    rel, rel_rounded, within2 = _accuracy(out, _fp64_reference(inp))
    if dtype == torch.float16:
        assert rel <= 1e-3, rel
    else:
        assert rel <= 8e-3 and rel_rounded <= 1e-3, (rel, rel_rounded)
    assert within2 >= 0.999, within2


@pytest.mark.parametrize(
    "m,n,k",
    [(1, 64, 64), (129, 64, 128), (128, 320, 320), (300, 192, 1088), (77, 576, 64), (256, 256, 2304),
     (8, 512, 1024), (16, 1024, 2048), (24, 768, 512)],
)
def test_edge_shapes_vs_oracle(cuda_ext, m, n, k):
    """Ragged M, N not a multiple of the 256-column tile, K tails of 1-3 scale blocks, and skinny M
    (fewer than 32 rows: the A box covers only the rows present)."""
    inp = _inputs(cuda_ext, m, n, k, seed=m + n + k)
    out = cuda_ext.gemm(inp["a"], inp["b"], inp["a_sf"], inp["b_sf"])
    c64 = oracle.gemm_fp64(*(inp[x].cpu().numpy() for x in ("a", "a_sf_linear", "b", "b_sf_linear")))
    rel, _, within2 = _accuracy(out, torch.from_numpy(c64).cuda())
    assert rel <= 1e-3 and within2 >= 0.999, (rel, within2)


@pytest.mark.parametrize(
    "cfg_kwargs",
    [
        dict(cluster=(4, 1), fallback=None, fast_swz=2, raster_along_m=False),
        dict(cluster=(8, 2), fallback=(2, 1), fast_swz=4, l2_policy_a="evict_last"),
        dict(cluster=(2, 2), fallback=None, epi_store_pace_per_ktile_ns=0),
        dict(tile=(128, 256), cluster=(1, 1), tma_b_first=True, l2_policy_b="evict_first"),
    ],
)
def test_configs(cuda_ext, cfg_kwargs):
    from gemm3_b200 import Config
    from gemm3_b200.testing import check, reference

    inp = _inputs(cuda_ext, 2048, 2048, 2048)
    out = cuda_ext.gemm(inp["a"], inp["b"], inp["a_sf"], inp["b_sf"], config=Config.make(**cfg_kwargs))
    ok, err = check(out, reference(inp))
    assert ok, err
    base = cuda_ext.gemm(inp["a"], inp["b"], inp["a_sf"], inp["b_sf"])
    assert torch.equal(out, base), "output bits depend on the launch configuration"


def test_fast_swz_falls_back_when_m_not_divisible(cuda_ext):
    from gemm3_b200 import Config
    from gemm3_b200.testing import check, reference

    cfg = Config.make(cluster=(4, 1), fallback=None, fast_swz=2)
    inp = _inputs(cuda_ext, 1536, 1024, 1024)
    with pytest.warns(UserWarning, match="fast_swz"):
        out = cuda_ext.gemm(inp["a"], inp["b"], inp["a_sf"], inp["b_sf"], config=cfg)
    ok, err = check(out, reference(inp))
    assert ok, err


def test_bf16_output(cuda_ext):
    from gemm3_b200.testing import check, reference

    inp = _inputs(cuda_ext, 1024, 1024, 1024)
    out = cuda_ext.gemm(inp["a"], inp["b"], inp["a_sf"], inp["b_sf"], out_dtype=torch.bfloat16)
    assert out.dtype == torch.bfloat16
    ok, err = check(out, reference(inp), rel_tol=8e-3)
    assert ok, err


def test_alpha_and_out_reuse(cuda_ext):
    inp = _inputs(cuda_ext, 512, 768, 1024)
    ref = _fp64_reference(inp, alpha=0.5)
    alpha = torch.tensor([0.5], device="cuda")
    c = torch.empty(512, 768, device="cuda", dtype=torch.bfloat16)
    out = cuda_ext.gemm(inp["a"], inp["b"], inp["a_sf"], inp["b_sf"], alpha=alpha, out=c, out_dtype=torch.bfloat16)
    assert out.data_ptr() == c.data_ptr()
    rel, rel_rounded, within2 = _accuracy(out, ref)
    assert rel_rounded <= 1e-3 and within2 >= 0.999
    with pytest.raises(ValueError):
        cuda_ext.gemm(inp["a"], inp["b"], inp["a_sf"], inp["b_sf"], out=c)  # dtype mismatch
    with pytest.raises(TypeError):
        cuda_ext.gemm(inp["a"], inp["b"], inp["a_sf"], inp["b_sf"], alpha=0.5)


def test_owned_8k_rejects_other_shapes(cuda_ext):
    from gemm3_b200 import config_for

    inp = _inputs(cuda_ext, 512, 512, 512)
    with pytest.raises(ValueError, match="M=N=K=8192"):
        cuda_ext.gemm(inp["a"], inp["b"], inp["a_sf"], inp["b_sf"], config=config_for(8192, 8192, 8192))


@pytest.mark.parametrize("size", [4096, 8192, 16384, 32768])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_presets_scaled_output(cuda_ext, size, dtype):
    """Every preset is bit-identical to a generic configuration (alpha = -0.375), and a
    size-independent property holds: C @ 1 equals alpha * A @ (B^T @ 1) in FP64."""
    from gemm3_b200 import Config, config_for, persisting_l2

    inp = _inputs(cuda_ext, size, size, size, seed=2)
    cfg = config_for(size, size, size)
    previous = Config.make(cluster=(8, 2), fallback=(2, 1), persist_mb=40, fast_swz=4, raster_along_m=False,
                           l2_policy_a="evict_last", l2_policy_sfa="evict_last")
    alpha = torch.tensor([-0.375], device="cuda", dtype=torch.float32)
    args = (inp["a"], inp["b"], inp["a_sf"], inp["b_sf"])
    with persisting_l2(cfg.persist_mb):
        expected = cuda_ext.gemm(*args, alpha=alpha, out_dtype=dtype, config=previous)
        actual = cuda_ext.gemm(*args, alpha=alpha, out_dtype=dtype, config=cfg)
    torch.testing.assert_close(actual, expected, rtol=0, atol=0)
    if size <= 16384:
        from gemm3_b200 import dequantize_nvfp4

        ones = torch.ones(size, 1, device="cuda", dtype=torch.float64)
        bsum = dequantize_nvfp4(inp["b"], inp["b_sf_linear"]).double().T @ ones
        rows = -0.375 * (dequantize_nvfp4(inp["a"], inp["a_sf_linear"]).double() @ bsum)
        got = actual.double() @ ones
        assert ((got - rows).norm() / rows.norm()).item() < 2e-3


def test_no_device_errors(cuda_ext):
    assert cuda_ext.device_status() == 0
