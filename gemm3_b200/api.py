"""Launch the B200 NVFP4 GEMM.

``gemm(a, b, a_sf, b_sf)`` computes ``C = alpha * dequant(A) @ dequant(B).T`` with A [M, K/2] and
B [N, K/2] packed NVFP4 (uint8, two values per byte) and scale factors in the 128x4 swizzled
layout (see ``quant.swizzle_sf``). Same signature, validation order and error messages as
nvfp4_gemm_cute/api.py:152-220; the launch goes to the hand-written sm_100a kernel in
libgemm3_b200.so through its C ABI, on the current torch stream, with no host synchronisation.
"""

import contextlib
import ctypes
import warnings

import torch

from . import _lib
from .hw import arch
from .presets import STREAM_MAX_M, config_for

_ALPHA_ONE = {}
_STATUS = {}
_CFG_CACHE = {}

_SUPPORTED_ATTRIBUTES = frozenset(
    {
        "fast_swz",
        "raster_along_m",
        "owned_8k",
        "l2_policy_a",
        "l2_policy_b",
        "l2_policy_sfa",
        "l2_policy_sfb",
        "epi_store_pace_per_ktile_ns",
        "prefetch_first_ktiles",
        "trim_short_tail",
        "tma_b_first",
        "tma_sfb_first",
        "retire_a_cols",
        "packed_ab_desc",
        "epi_store_pair",
        "specialize_32k",
    }
)

_L2_POLICIES = {
    None: _lib.L2_NORMAL,
    "evict_normal": _lib.L2_NORMAL,
    "evict_first": _lib.L2_EVICT_FIRST,
    "evict_last": _lib.L2_EVICT_LAST,
}

_OUT_DTYPES = {torch.float16: _lib.DTYPE_F16, torch.bfloat16: _lib.DTYPE_BF16}


def supported() -> bool:
    """Return True if the current GPU is sm_100 (B200/GB200) and the extension loads."""
    if not torch.cuda.is_available() or arch() != "sm_100":
        return False
    try:
        _lib.lib()
    except (OSError, RuntimeError):
        return False
    return True


def _out_code(dtype):
    if dtype not in _OUT_DTYPES:
        raise ValueError(f"unsupported output dtype {dtype}; use float16 or bfloat16")
    return _OUT_DTYPES[dtype]


def _num_m_clusters(m, cfg):
    cta_m = 128  # 2-CTA 256-row tiles and 1-CTA 128-row tiles both use 128-row CTA tiles
    return -(-(-(-m // cta_m)) // cfg.cluster[0])


def _effective_attrs(m, cfg):
    """Return the kernel attributes for this launch, with fast_swz dropped if M does not allow it.

    fast_swz groups fast_swz M-clusters into one raster band (nvfp4_gemm_cute/api.py:67-89); when
    the M-cluster count is not a multiple of it the reference falls back to plain raster order,
    and so does this module.
    """
    attrs = cfg.attr_dict()
    unknown = set(attrs) - _SUPPORTED_ATTRIBUTES
    if unknown:
        raise ValueError(f"unsupported kernel attributes: {', '.join(sorted(unknown))}")
    s = attrs.get("fast_swz", 1)
    if s > 1:
        if s & (s - 1):
            raise ValueError(f"fast_swz must be a power of two, got {s}")
        if _num_m_clusters(m, cfg) % s:
            warnings.warn(
                f"fast_swz={s} needs the M-cluster count ({_num_m_clusters(m, cfg)}) to be a "
                "multiple of it; falling back to plain raster order",
                stacklevel=3,
            )
            attrs["fast_swz"] = 1
        attrs["raster_along_m"] = False
    return attrs


def _check_shape_guards(m, n, k, cfg, attrs):
    """Shape/cluster guards of the specialised presets (nvfp4_gemm_cute/api.py:177-207)."""
    if attrs.get("specialize_32k"):
        if (m, n, k) != (32768, 32768, 32768):
            raise ValueError("32K specialization requires M=N=K=32768")
        if cfg.tile != (256, 256) or cfg.cluster != (4, 4) or cfg.fallback != (2, 1):
            raise ValueError(
                "32K specialization requires tile=(256, 256), cluster=(4, 4), fallback=(2, 1)"
            )
    if attrs.get("owned_8k") and (m, n, k) != (8192, 8192, 8192):
        raise ValueError("owned_8k scheduling requires M=N=K=8192")
    if attrs.get("owned_8k") and (
        cfg.tile != (256, 256) or cfg.cluster != (8, 2) or cfg.fallback != (2, 1)
    ):
        raise ValueError(
            "owned_8k scheduling requires tile=(256, 256), cluster=(8, 2), fallback=(2, 1)"
        )
    if attrs.get("trim_short_tail"):
        if (m, n, k) != (16384, 16384, 16384):
            raise ValueError("16K optimizations require M=N=K=16384")
        if cfg.tile != (256, 256) or cfg.cluster != (8, 2) or cfg.fallback != (2, 1):
            raise ValueError(
                "16K optimizations require tile=(256, 256), cluster=(8, 2), fallback=(2, 1)"
            )
    if attrs.get("packed_ab_desc"):
        expected_cluster = {(16384, 16384, 16384): (8, 2), (32768, 32768, 32768): (4, 4)}
        cluster = expected_cluster.get((m, n, k))
        if cluster is None:
            raise ValueError("packed_ab_desc requires M=N=K=16384 or M=N=K=32768")
        if cfg.tile != (256, 256) or cfg.cluster != cluster or cfg.fallback != (2, 1):
            raise ValueError(
                f"packed_ab_desc requires tile=(256, 256), cluster={cluster}, fallback=(2, 1)"
            )
    if cfg.tile not in ((256, 256), (128, 256), (128, 128)):
        raise ValueError(f"unsupported tile {cfg.tile}; use (256, 256), (128, 256) or (128, 128)")
    if cfg.tile == (128, 128) and m > STREAM_MAX_M:
        raise ValueError(
            f"tile (128, 128) streams B with all of A's rows in one tile and needs M <= {STREAM_MAX_M} "
            f"(got M={m})"
        )


def _launch_config(m, k, cfg, attrs, pdl=0):
    """Translate a Config + effective attributes into the C struct (cached)."""
    key = (m, k, cfg.tile, cfg.cluster, tuple(sorted(attrs.items())), pdl)
    c = _CFG_CACHE.get(key)
    if c is not None:
        return c
    c = _lib.GemmConfig()
    c.struct_size = ctypes.sizeof(_lib.GemmConfig)
    # 256: CTA-pair kernel; 128: one CTA per 128x256 tile; (128, 128): weight-streaming kernel
    c.tile_m = 256 if cfg.tile[0] == 256 else 128
    c.tile_n = cfg.tile[1]
    c.pdl = pdl
    m_tiles = -(-m // 128)
    s = int(attrs.get("fast_swz", 1) or 1)
    if s > 1:
        band = s * max(1, int(cfg.cluster[0])) * (cfg.tile[0] // 128)
    else:
        band = m_tiles  # plain M-fast raster: one band spanning every M tile
    c.raster_band = max(1, min(band, m_tiles))
    c.raster_along_m = 0
    for field in ("a", "b", "sfa", "sfb"):
        pol = attrs.get(f"l2_policy_{field}")
        if pol not in _L2_POLICIES:
            raise ValueError(f"unsupported l2_policy_{field} {pol!r}")
        setattr(c, f"l2_policy_{field}", _L2_POLICIES[pol])
    c.store_evict_first = 0
    pace = int(attrs.get("epi_store_pace_per_ktile_ns", 0) or 0)
    c.epi_store_pace_ns = pace * (-(-k // 768)) if pace > 0 else 0
    c.tma_b_first = 1 if attrs.get("tma_b_first") else 0
    c.max_ctas = 0
    _CFG_CACHE[key] = c
    return c


def _status_word(dev):
    st = _STATUS.get(dev)
    if st is None:
        st = _STATUS[dev] = torch.zeros(1, dtype=torch.int32, device=dev)
    return st


def device_status(device=None, reset=True) -> int:
    """Synchronise ``device`` and return the first device-side error code recorded by a kernel
    launched through this module (0 = none); ``reset`` clears it."""
    dev = torch.device("cuda", torch.cuda.current_device() if device is None else torch.device(device).index)
    st = _STATUS.get(dev)
    if st is None:
        return 0
    code = int(st.item())
    if reset and code:
        st.zero_()
    return code


def gemm(
    a, b, a_sf, b_sf, alpha=None, out=None, out_dtype=torch.float16, config=None, enable_pdl=True
):
    """Compute ``alpha * dequant(a) @ dequant(b).T`` on sm_100.

    Args:
        a: [M, K/2] uint8 packed NVFP4 (row-major, K contiguous).
        b: [N, K/2] uint8 packed NVFP4 (the weight layout, K contiguous).
        a_sf, b_sf: E4M3 scale factors in the 128x4 swizzled layout (uint8 or float8_e4m3fn).
        alpha: optional float32 tensor with one element; defaults to 1.0.
        out: optional [M, N] output of out_dtype.
        config: a presets.Config; defaults to presets.config_for(M, N, K).
        enable_pdl: launch with programmatic dependent launch (nvfp4_gemm_cute/kernel.py:524):
            the kernel's set-up (barriers, TMEM, tensor-map prefetch) overlaps the tail of the
            preceding kernel on the stream, and it reads and writes global memory only after
            that kernel has completed. This holds for every kernel (CTA-pair, one-CTA,
            weight-streaming); the CTA-pair and one-CTA kernels also let the next PDL launch on
            the stream start its set-up as soon as SMs free up.

    Requires N % 64 == 0 and K % 64 == 0. Shape, attribute and preset checks raise ValueError
    before any GPU work.
    """
    return _gemm(a, b, a_sf, b_sf, alpha, out, out_dtype, config, 1 if enable_pdl else 0)


def _gemm(a, b, a_sf, b_sf, alpha, out, out_dtype, config, pdl):
    """gemm() with the C config's programmatic-dependent-launch mode (0, 1 or 2; see
    include/nvfp4_gemm.h). Mode 2 (weights loaded before the dependency wait) is for callers that
    know the preceding kernel does not write B, such as linear.nvfp4_linear."""
    m, kp = a.shape
    n = b.shape[0]
    k = kp * 2
    if b.shape[1] != kp:
        raise ValueError(f"K mismatch: a is [{m}, {kp}], b is [{n}, {b.shape[1]}]")
    if n % 64 or k % 64:
        raise ValueError(f"N and K must be multiples of 64 (got N={n}, K={k})")
    cfg = config or config_for(m, n, k)
    attrs = _effective_attrs(m, cfg)
    _check_shape_guards(m, n, k, cfg, attrs)
    code = _out_code(out_dtype)
    ccfg = _launch_config(m, k, cfg, attrs, pdl)

    dev = a.device
    if dev.type != "cuda":
        raise ValueError("gemm needs CUDA tensors")
    for name, t in (("b", b), ("a_sf", a_sf), ("b_sf", b_sf)):
        if t.device != dev:
            raise ValueError(f"{name} is on {t.device}, a is on {dev}")
    if a.dtype != torch.uint8 or b.dtype != torch.uint8:
        raise ValueError("a and b must be uint8 packed NVFP4")
    if not (a.is_contiguous() and b.is_contiguous()):
        raise ValueError("a and b must be contiguous")
    for name, t, rows in (("a_sf", a_sf, m), ("b_sf", b_sf, n)):
        if t.dtype not in (torch.uint8, torch.float8_e4m3fn) or not t.is_contiguous():
            raise ValueError(f"{name} must be a contiguous uint8 or float8_e4m3fn tensor")
        need = -(-rows // 128) * 128 * (-(-k // 64)) * 4
        if t.numel() < need:
            raise ValueError(f"{name} has {t.numel()} scale bytes, needs {need}")
        if t.data_ptr() % 16:
            raise ValueError(f"{name} must be 16-byte aligned")
    if out is None:
        out = torch.empty(m, n, dtype=out_dtype, device=dev)
    else:
        if out.dtype != out_dtype:
            raise ValueError(f"out has dtype {out.dtype}, expected out_dtype={out_dtype}")
        if tuple(out.shape) != (m, n) or not out.is_contiguous():
            raise ValueError(f"out must be a contiguous [{m}, {n}] tensor")
        if out.data_ptr() % 32:
            raise ValueError("out must be 32-byte aligned")
        if out.device != dev:
            raise ValueError(f"out is on {out.device}, a is on {dev}")
    if alpha is None:
        alpha = _ALPHA_ONE.get(dev)
        if alpha is None:
            alpha = _ALPHA_ONE[dev] = torch.ones(1, dtype=torch.float32, device=dev)
    else:
        if not isinstance(alpha, torch.Tensor) or alpha.numel() != 1:
            raise TypeError("alpha must be a one-element CUDA tensor")
        alpha = alpha.reshape(1).to(device=dev, dtype=torch.float32)
    status = _status_word(dev)
    L = _lib.lib()
    with torch.cuda.device(dev):
        stream = torch.cuda.current_stream(dev).cuda_stream
        rc = L.nvfp4_gemm_run(
            a.data_ptr(), b.data_ptr(), a_sf.data_ptr(), b_sf.data_ptr(), out.data_ptr(),
            alpha.data_ptr(), m, n, k, code, ctypes.byref(ccfg), status.data_ptr(), stream,
        )
    _lib.check(rc, "nvfp4_gemm_run")
    return out


@contextlib.contextmanager
def persisting_l2(mb: int):
    """Set the persisting-L2 limit to ``mb`` MiB for this scope, then restore the old limit.

    This host limit (cudaLimitPersistingL2CacheSize) belongs to the process's CUDA context; it
    does not select addresses or guarantee residency. Restoration happens on context exit and
    does not synchronize with GPU completion. Nothing is changed when the limit already has the
    requested value.
    """
    torch.cuda.init()
    L = _lib.lib()
    old = ctypes.c_int64(0)
    want = int(mb) << 20
    _lib.check(L.nvfp4_set_persisting_l2(want, ctypes.byref(old)), f"persisting_l2({mb} MB)")
    try:
        yield
    finally:
        if old.value != want:
            L.nvfp4_set_persisting_l2(old.value, ctypes.byref(ctypes.c_int64(0)))
