"""Per-shape launch configurations for the B200 (sm_100a) NVFP4 GEMM.

Same interface as nvfp4_gemm_cute/presets.py:14-99: a frozen ``Config`` (tile, preferred cluster,
fallback cluster, sorted attribute tuple, persisting-L2 MiB), ``DEFAULT``, ``PRESETS`` keyed by
(M, N, K) and ``config_for``.

How the fields act on the B200 kernels (gemm3_b200/csrc/gemm_pair_kernel.cuh, gemm_kernel.cuh):
  tile            (256, 256): CTA pairs (tcgen05 cta_group::2), one 256x256 tile per pair;
                  (128, 256): one CTA per 128x256 tile. The accumulation order, and so the output
                  bits, are the same for every tile, cluster, raster and cache setting.
  cluster         kept for the tile order: ``fast_swz`` groups tiles in bands of
                  fast_swz * cluster[0] CTA tiles along M. The B200 kernel uses no TMA multicast,
                  so cluster shape does not change data movement.
  fallback        accepted and validated; unused (no multicast cluster to fall back from).
  persist_mb      host persisting-L2 limit to hold while calling (``api.persisting_l2``).
Measured on B200 (python -m gemm3_b200.tune, BF16 out; outputs bit-identical across all):
  - the CTA-pair tile beats the one-CTA tile at every size (8192^3: 215 against 371 us; the
    one-CTA tile reads 42 % more from L2);
  - at 16384^3 the fast_swz=2 band with cluster (8, 2) is 12-21 % faster than plain raster, raster
    along M, or fast_swz 1, 4 or 8 (1536 against 1740-1975 us): it keeps the B tiles in sweep
    resident in L2; A/SFA evict_last adds 1 % and B evict_first 2.6 %;
  - at 32768^3 the band of fast_swz=2 with cluster (4, 4) beats fast_swz=4 by 5 % (14.1 against
    14.9 ms) and B evict_first adds 3.5 %;
  - at 8192^3 and 4096^3 (operands resident in L2) raster and L2 attributes change the time by at
    most one 2-us timer step.
Attributes with an effect: fast_swz, raster_along_m, l2_policy_{a,b,sfa,sfb},
epi_store_pace_per_ktile_ns, tma_b_first. The others (owned_8k, trim_short_tail, tma_sfb_first,
retire_a_cols, packed_ab_desc, epi_store_pair, specialize_32k, prefetch_first_ktiles) name
B300 code paths of the reference kernel; they are accepted and shape-checked with the same
rules and messages as the reference (nvfp4_gemm_cute/api.py:177-207) and do not change the B200
kernel.
"""

from dataclasses import dataclass, field


@dataclass(frozen=True)
class Config:
    """Launch configuration for one GEMM shape."""

    tile: tuple = (256, 256)
    cluster: tuple = (4, 1)
    fallback: tuple | None = (2, 1)
    attrs: tuple = field(default_factory=tuple)  # sorted ((name, value), ...)
    persist_mb: int = 0

    @staticmethod
    def make(tile=(256, 256), cluster=(4, 1), fallback=(2, 1), persist_mb=0, **attrs):
        return Config(
            tuple(tile),
            tuple(cluster),
            fallback and tuple(fallback),
            tuple(sorted(attrs.items())),
            persist_mb,
        )

    def attr_dict(self):
        return dict(self.attrs)


# General-purpose default: plain raster order, standard L2 policy.
DEFAULT = Config.make()

# (M, N, K) -> Config. Shape-specific attributes keep the reference's guards; the B200 knobs are
# the raster band (fast_swz x cluster[0] CTA tiles) and the operand L2 policies.
PRESETS = {
    (4096, 4096, 4096): Config.make(
        cluster=(4, 2),
        fallback=(2, 1),
        fast_swz=2,
        raster_along_m=False,
        prefetch_first_ktiles=1,
    ),
    (8192, 8192, 8192): Config.make(
        cluster=(8, 2),
        fallback=(2, 1),
        fast_swz=2,
        raster_along_m=False,
        owned_8k=True,
        l2_policy_a="evict_last",
        l2_policy_sfa="evict_last",
    ),
    (16384, 16384, 16384): Config.make(
        cluster=(8, 2),
        fallback=(2, 1),
        fast_swz=2,
        raster_along_m=False,
        l2_policy_a="evict_last",
        l2_policy_sfa="evict_last",
        l2_policy_b="evict_first",
        trim_short_tail=True,
        tma_b_first=True,
        tma_sfb_first=True,
        retire_a_cols=8,
        packed_ab_desc=True,
    ),
    (32768, 32768, 32768): Config.make(
        cluster=(4, 4),
        fallback=(2, 1),
        fast_swz=2,
        raster_along_m=False,
        l2_policy_a="evict_last",
        l2_policy_b="evict_first",
        epi_store_pair=True,
        epi_store_pace_per_ktile_ns=0,
        retire_a_cols=8,
        packed_ab_desc=True,
        specialize_32k=True,
    ),
}

# B200 additions: the per-GPU shapes of the N-sharded 32768^3 scaling run (N / 8, N / 4, N / 2 per
# rank). A band of 8 CTA tiles (4 CTA-pair tiles) along M keeps the pairs in flight on the same
# A rows while every B tile of the rank's slice stays in L2; plain raster re-streams A (17-19 %
# slower). Keeping A resident (evict_last) and streaming B (evict_first) adds 2-5 %.
for _n in (4096, 8192, 16384):
    PRESETS[(32768, _n, 32768)] = Config.make(
        cluster=(4, 1),
        fallback=(2, 1),
        fast_swz=2,
        raster_along_m=False,
        l2_policy_a="evict_last",
        l2_policy_sfa="evict_last",
        l2_policy_b="evict_first",
    )
del _n


# B200 retune for skinny GEMMs (M <= 128, e.g. LLM projections on a few tokens): the
# weight-streaming kernel, tile (128, 128). B's rows fill the tensor core's M dimension in 128-row
# tiles and all of A's rows form its N, so every SM streams its own rows of B once (N/128 tiles
# instead of N/256) and no MMA work goes to absent rows of A. The one-CTA 128x256 tile
# (tile=(128, 256)) remains available; a 256-row CTA-pair tile would be at least half empty.
STREAM_MAX_M = 128
SKINNY = Config.make(tile=(128, 128))
SKINNY_MAX_M = STREAM_MAX_M


def config_for(m: int, n: int, k: int) -> Config:
    """Return the tuned configuration for (m, n, k): a preset, SKINNY for M <= 128, else DEFAULT."""
    cfg = PRESETS.get((m, n, k))
    if cfg is not None:
        return cfg
    return SKINNY if m <= SKINNY_MAX_M else DEFAULT
