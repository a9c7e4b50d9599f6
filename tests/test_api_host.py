"""CPU: host-side behaviour of the drop-in API — validation before any GPU work, with the
reference's messages (nvfp4_gemm_cute tests/test_gemm.py:51-142, api.py:67-207)."""

import ctypes
from dataclasses import replace

import pytest
import torch

import gemm3_b200 as g3
from gemm3_b200 import Config, config_for
from gemm3_b200.api import _effective_attrs, _launch_config


def _expanded(rows, cols):
    # Validation happens before compilation or GPU access; expanded views avoid large allocations.
    return torch.empty(1, dtype=torch.uint8).expand(rows, cols)


SF = torch.empty(1, dtype=torch.uint8)


def test_public_api_matches_reference_exports():
    for name in ("DEFAULT", "PRESETS", "Config", "config_for", "dequantize_nvfp4", "gemm", "persisting_l2",
                 "quantize_nvfp4", "supported", "swizzle_sf"):
        assert hasattr(g3, name), name


def test_config_make_and_presets():
    c = Config.make(cluster=(8, 2), fast_swz=4, l2_policy_a="evict_last")
    assert c.tile == (256, 256) and c.cluster == (8, 2) and c.fallback == (2, 1)
    assert c.attrs == (("fast_swz", 4), ("l2_policy_a", "evict_last"))
    assert Config.make(fallback=None).fallback is None
    assert config_for(1024, 2048, 4096) == g3.DEFAULT
    assert config_for(16, 28672, 8192).tile == (128, 128)  # B200 weight-streaming kernel for M <= 128
    assert config_for(129, 28672, 8192) == g3.DEFAULT
    for size in (4096, 8192, 16384, 32768):
        assert config_for(size, size, size) is g3.PRESETS[(size, size, size)]


def test_k_mismatch():
    with pytest.raises(ValueError, match="K mismatch"):
        g3.gemm(_expanded(128, 64), _expanded(128, 32), SF, SF)


@pytest.mark.parametrize("n,kp", [(100, 64), (128, 48)])
def test_n_k_multiples_of_64(n, kp):
    with pytest.raises(ValueError, match="N and K must be multiples of 64"):
        g3.gemm(_expanded(128, kp), _expanded(n, kp), SF, SF)


def test_owned_8k_rejects_other_shapes():
    with pytest.raises(ValueError, match="M=N=K=8192"):
        g3.gemm(_expanded(512, 256), _expanded(512, 256), SF, SF, config=config_for(8192, 8192, 8192))


def test_16k_preset_rejects_other_shapes():
    with pytest.raises(ValueError, match="M=N=K=16384"):
        g3.gemm(_expanded(512, 256), _expanded(512, 256), SF, SF, config=config_for(16384, 16384, 16384))


@pytest.mark.parametrize(
    "overrides, message",
    [
        ({"cluster": (4, 1)}, "cluster="),
        ({"attrs": (("packed_ab_desc", True), ("swap_ab", True))}, "unsupported kernel attributes"),
    ],
)
def test_16k_preset_rejects_incompatible_config(overrides, message):
    a = _expanded(16384, 8192)
    cfg = replace(config_for(16384, 16384, 16384), **overrides)
    with pytest.raises(ValueError, match=message):
        g3.gemm(a, a, SF, SF, config=cfg)


@pytest.mark.parametrize("overrides,message", [({"shape": 512}, "M=N=K=32768"), ({"cluster": (8, 2)}, "cluster=")])
def test_32k_preset_guards(overrides, message):
    size = overrides.get("shape", 32768)
    a = _expanded(size, size // 2)
    cfg = config_for(32768, 32768, 32768)
    if "cluster" in overrides:
        cfg = replace(cfg, cluster=overrides["cluster"])
    with pytest.raises(ValueError, match=message):
        g3.gemm(a, a, SF, SF, config=cfg)


def test_unsupported_output_dtype():
    with pytest.raises(ValueError, match="unsupported output dtype"):
        g3.gemm(_expanded(128, 64), _expanded(128, 64), SF, SF, out_dtype=torch.float32)


def test_fast_swz_must_be_power_of_two():
    with pytest.raises(ValueError, match="fast_swz must be a power of two"):
        _effective_attrs(4096, Config.make(fast_swz=3))


def test_fast_swz_fallback_warning_and_raster_band():
    # 3 M-clusters of 4x1 (M=1536) cannot be grouped by fast_swz=2.
    cfg = Config.make(cluster=(4, 1), fallback=None, fast_swz=2)
    with pytest.warns(UserWarning, match="fast_swz"):
        attrs = _effective_attrs(1536, cfg)
    assert attrs["fast_swz"] == 1 and attrs["raster_along_m"] is False
    # plain raster: one band spanning all 128-row tiles
    assert _launch_config(1536, 1024, cfg, attrs).raster_band == 12
    attrs = _effective_attrs(2048, cfg)
    assert _launch_config(2048, 1024, cfg, attrs).raster_band == 2 * 4 * 2


def test_l2_policy_names():
    cfg = Config.make(l2_policy_a="evict_last", l2_policy_b="evict_first")
    c = _launch_config(256, 256, cfg, _effective_attrs(256, cfg))
    assert (c.l2_policy_a, c.l2_policy_b, c.l2_policy_sfa) == (2, 1, 0)
    bad = Config.make(l2_policy_a="keep")
    with pytest.raises(ValueError, match="l2_policy_a"):
        _launch_config(256, 256, bad, _effective_attrs(256, bad))


def test_cpu_operands_rejected_after_guards():
    with pytest.raises(ValueError, match="CUDA"):
        g3.gemm(_expanded(128, 64), _expanded(128, 64), SF, SF)


def test_stream_tile_needs_skinny_m():
    """tile (128, 128) (weight-streaming kernel) holds all of A's rows in one MMA: M <= 128."""
    a = torch.empty(1, dtype=torch.uint8).expand(129, 64)
    b = torch.empty(1, dtype=torch.uint8).expand(128, 64)
    sf = torch.empty(1, dtype=torch.uint8)
    with pytest.raises(ValueError, match="M <= 128"):
        g3.gemm(a, b, sf, sf, config=Config.make(tile=(128, 128)))
    with pytest.raises(ValueError, match="unsupported tile"):
        g3.gemm(a, b, sf, sf, config=Config.make(tile=(64, 128)))


def test_quantize_act_validation_before_gpu():
    from gemm3_b200 import _lib, build

    build.build()
    L = _lib.lib()
    p = ctypes.c_void_p(1 << 20)  # never dereferenced: validation answers first
    assert L.nvfp4_quantize_act(p, 1, 4, 24, None, None, None, p, p, p, None) == _lib.ERR_INVALID_VALUE  # K % 16
    # alpha needs the other operand's global scale; the workspace is required
    assert L.nvfp4_quantize_act(p, 1, 4, 64, None, None, p, p, p, p, None) == _lib.ERR_INVALID_VALUE
    assert L.nvfp4_quantize_act(p, 1, 4, 64, None, None, None, p, p, None, None) == _lib.ERR_INVALID_VALUE
    assert L.nvfp4_quantize_act(p, 1, 4, 64, None, None, None, p, p, ctypes.c_void_p((1 << 20) + 2), None) == (
        _lib.ERR_MISALIGNED
    )
