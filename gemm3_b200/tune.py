"""Time the GEMM over launch configurations for one shape, as evidence for a preset.

    python -m gemm3_b200.tune --size 8192 [--shape M N K ...] [--out-dtype bfloat16] [--iters 40]
                              [--markdown file.md]

For M = N = K = size (and for each --shape) it times the preset of ``presets.config_for`` and
variants of it that change one B200 knob at a time (tile, raster band, raster direction, operand
L2 policies, a persisting-L2 reservation, TMA issue order), with the timing of
``compare.time_us``: the median of CUDA-event samples around one CUDA-graph replay, after an L2
flush. Every variant's output is compared bit for bit with the preset's: the accumulation order
does not depend on the configuration. One JSON line per configuration; ``--markdown`` also
writes the table.
"""

import argparse
import json
from pathlib import Path

import torch

from . import api, compare, presets, testing

# Attributes that act on the B200 kernels (the others only carry the reference's shape guards).
_ACTIVE = ("fast_swz", "raster_along_m", "l2_policy_a", "l2_policy_b", "l2_policy_sfa", "l2_policy_sfb",
           "epi_store_pace_per_ktile_ns", "tma_b_first")


def active_attrs(cfg):
    return {k: v for k, v in cfg.attr_dict().items() if k in _ACTIVE}


def candidates(m, n, k):
    """(name, Config) pairs: the preset, the plain default, and one-knob variants of the preset."""
    base = presets.config_for(m, n, k)
    attrs = active_attrs(base)
    cluster = base.cluster
    out = [("preset", base), ("default", presets.DEFAULT)]

    def variant(name, tile=(256, 256), clu=cluster, persist_mb=0, **changes):
        a = dict(attrs)
        for k_, v in changes.items():
            if v is None:
                a.pop(k_, None)
            else:
                a[k_] = v
        out.append((name, presets.Config.make(tile=tile, cluster=clu, fallback=(2, 1), persist_mb=persist_mb, **a)))

    variant("tile (128, 256)", tile=(128, 256))
    m_clusters = -(-m // 128) // cluster[0]
    for s in (1, 2, 4, 8):
        if s != attrs.get("fast_swz", 1) and m_clusters % s == 0:
            variant(f"fast_swz={s}", fast_swz=s, raster_along_m=False)
    variant("raster along M", fast_swz=None, raster_along_m=True)
    if attrs.get("l2_policy_a") == "evict_last":
        variant("A and SFA evict_normal", l2_policy_a=None, l2_policy_sfa=None)
    else:
        variant("A and SFA evict_last", l2_policy_a="evict_last", l2_policy_sfa="evict_last")
    variant("A and SFA evict_last, persisting L2 48 MiB", persist_mb=48, l2_policy_a="evict_last",
            l2_policy_sfa="evict_last")
    if attrs.get("l2_policy_b") == "evict_first":
        variant("B evict_normal", l2_policy_b=None)
    else:
        variant("B evict_first", l2_policy_b="evict_first")
    variant("B loads first" if not attrs.get("tma_b_first") else "A loads first",
            tma_b_first=not attrs.get("tma_b_first"))
    return out


def run(m, n, k, out_dtype, iters):
    inp = testing.make_inputs(m, n, k, seed=0)
    flops = 2.0 * m * n * k
    ref = None
    rows = []
    for name, cfg in candidates(m, n, k):
        out = torch.empty((m, n), device="cuda", dtype=out_dtype)

        def call(cfg=cfg, out=out):
            api.gemm(inp["a"], inp["b"], inp["a_sf"], inp["b_sf"], out=out, out_dtype=out_dtype, config=cfg)

        with api.persisting_l2(cfg.persist_mb):
            us = compare.time_us(call, iters=iters)
        if ref is None:
            ref = out.clone()
        size = m if m == n == k else f"{m}x{n}x{k}"
        row = dict(size=size, config=name, tile=list(cfg.tile), cluster=list(cfg.cluster), attrs=active_attrs(cfg),
                   persist_mb=cfg.persist_mb, us=round(us, 2), pflops=round(flops / us / 1e9, 3),
                   bit_identical=bool(torch.equal(out, ref)))
        print(json.dumps(row), flush=True)
        rows.append(row)
        del out
    assert api.device_status() == 0
    return rows


def markdown(rows):
    lines = ["| size | configuration | tile | active attributes | persist MiB | µs | PFLOP/s | bits = preset |",
             "|---:|---|---|---|---:|---:|---:|---|"]
    for r in rows:
        attrs = ", ".join(f"{k}={v}" for k, v in sorted(r["attrs"].items())) or "—"
        lines.append(f"| {r['size']} | {r['config']} | {tuple(r['tile'])} | {attrs} | {r.get('persist_mb', 0)} | "
                     f"{r['us']:.1f} | {r['pflops']:.2f} | {'yes' if r['bit_identical'] else 'NO'} |")
    return "\n".join(lines) + "\n"


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--size", type=int, nargs="*", default=[])
    ap.add_argument("--shape", type=int, nargs=3, action="append", default=[], metavar=("M", "N", "K"))
    ap.add_argument("--out-dtype", default="bfloat16", choices=["float16", "bfloat16"])
    ap.add_argument("--iters", type=int, default=40)
    ap.add_argument("--markdown", type=Path)
    args = ap.parse_args(argv)
    assert api.supported(), "needs an sm_100 GPU and the built extension"
    shapes = [(s_, s_, s_) for s_ in args.size] + [tuple(x) for x in args.shape]
    if not shapes:
        ap.error("give --size and/or --shape")
    rows = []
    for m, n, k in shapes:
        rows += run(m, n, k, getattr(torch, args.out_dtype), args.iters)
    if args.markdown:
        args.markdown.write_text(markdown(rows))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
