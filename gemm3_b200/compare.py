"""Compare NVFP4 GEMM implementations on identical quantized inputs, on one B200.

The B200 counterpart of the reference's benchmark harness (benchmarks/compare.py, timing from
benchmarks/harness.py, figures from figures/plot.py):

    python -m gemm3_b200.compare run --size 8192 --rounds 8 --output results/compare-8192.json
    python -m gemm3_b200.compare summary results/compare-*.json --markdown table.md --svg plot.svg

`run` quantises one set of inputs (testing.make_inputs, seed 0), checks this package's output for
both output dtypes against an FP32 product of dequantised rows and columns sampled across the
whole output (compare.py:189-197), then validates every other implementation against this
package's output (bit equality and relative L2 with the reference's thresholds, compare.py:154-169)
and times all of them in rotated rounds: round r starts at implementation r mod n and runs the
order backwards on odd rounds (compare.py:271-274). Before and after every measurement the set of
processes on the GPU is compared with the one at the start; a change aborts the run
(compare.py:200-214). The JSON written after every step holds the samples, medians, checks,
device, source SHA-256 hashes and the GPU libraries the process loaded (compare.py:216-253).

Implementations: `preset` (gemm3_b200.gemm with presets.config_for), `cublaslt` (cuBLASLt through
libgemm3_b200_cublaslt.so) and, when FlashInfer can build them here, `cutlass`, `cudnn` and
`cute-dsl` (flashinfer.mm_fp4, as in compare.py:143-162). An implementation that fails to set up
or validate is recorded under "errors", as in the reference.

Timing differs from the reference in one respect, recorded in the JSON: the reference reads
kernel durations from CUPTI, which is not installed here, so each sample is a CUDA-event pair
around one replay of a CUDA graph holding the call, after an L2 flush (a write of twice the L2
size) and followed by a cooldown sleep, as in harness.py (cold L2, graph replay, sleep after run).
"""

import argparse
import hashlib
import json
import os
import statistics
import subprocess
import time
from pathlib import Path

PKG = Path(__file__).resolve().parent
SOURCES = [
    *sorted((PKG / "csrc").glob("*.cu*")),
    *(PKG / name for name in ("api.py", "presets.py", "quant.py", "compare.py")),
    *sorted((PKG.parent / "include").glob("*.h")),
]
LIBRARIES = ["preset", "cublaslt", "cutlass", "cudnn", "cute-dsl"]
LABELS = {
    "preset": "gemm3_b200 (this package)",
    "cublaslt": "cuBLASLt",
    "cutlass": "CUTLASS (FlashInfer)",
    "cudnn": "cuDNN (FlashInfer)",
    "cute-dsl": "FlashInfer CuTe DSL",
}
# relative L2 bounds of the reference (compare.py:161-162)
TOLERANCE = {"torch.bfloat16": 0.003, "torch.float16": 0.0005}


def rotated_order(names, rnd):
    """Round `rnd` (0-based) starts at names[rnd % n]; odd rounds run backwards."""
    k = rnd % len(names)
    order = names[k:] + names[:k]
    return order[::-1] if rnd % 2 else order


def source_hashes(root=PKG.parent):
    return {str(p.relative_to(root)): hashlib.sha256(p.read_bytes()).hexdigest() for p in SOURCES if p.exists()}


def time_us(fn, iters=50, cooldown_s=0.001):
    """Median over `iters` samples of one CUDA-graph replay of `fn`, cold L2, in microseconds."""
    import torch

    dev = torch.cuda.current_device()
    l2 = torch.cuda.get_device_properties(dev).L2_cache_size
    flush = torch.empty(2 * l2, dtype=torch.uint8, device="cuda")
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        fn()  # warm-up outside the capture (first-call set-up)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            fn()
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    samples = []
    for i in range(max(3, iters // 4) + iters):
        flush.fill_(i & 0xFF)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        g.replay()
        e1.record()
        e1.synchronize()
        if i >= max(3, iters // 4):
            samples.append(e0.elapsed_time(e1) * 1e3)
        time.sleep(cooldown_s)
    del g
    return statistics.median(samples)


def accuracy(out, ref):
    """Relative L2, bit equality and finiteness of out against ref, in 128-row chunks
    (compare.py:165-182); raises when the relative L2 exceeds the reference's bound."""
    import torch

    sqerr = torch.zeros((), device="cuda", dtype=torch.float64)
    sqref = torch.zeros_like(sqerr)
    exact, finite = True, True
    for start in range(0, out.shape[0], 128):
        a, b = out[start : start + 128].float(), ref[start : start + 128].float()
        sqerr += (a - b).square().sum(dtype=torch.float64)
        sqref += b.square().sum(dtype=torch.float64)
        exact = exact and torch.equal(a, b)
        finite = finite and bool(torch.isfinite(a).all())
    rel = (sqerr / sqref).sqrt().item()
    if not finite or rel > TOLERANCE[str(out.dtype)]:
        raise RuntimeError(f"numerical check failed: relative L2={rel}, finite={finite}")
    return dict(bit_exact=exact, relative_l2=rel, finite=finite)


def adapter(name, inp, size, out_dtype):
    """Return (run, out, metadata, keepalive) for one implementation at M = N = K = size."""
    import torch

    import gemm3_b200 as g3

    m = n = k = size
    out = torch.empty((m, n), device="cuda", dtype=out_dtype)
    meta, keep = {}, []
    if name == "preset":
        cfg = g3.config_for(m, n, k)
        meta["config"] = dict(tile=cfg.tile, cluster=cfg.cluster, attrs=cfg.attr_dict())

        def run():
            g3.gemm(inp["a"], inp["b"], inp["a_sf"], inp["b_sf"], out=out, out_dtype=out_dtype, config=cfg)

    elif name == "cublaslt":
        from gemm3_b200 import cublaslt

        def run():
            cublaslt.gemm_cublaslt(inp["a"], inp["b"], inp["a_sf"], inp["b_sf"], out=out, out_dtype=out_dtype)

        meta["library"] = "cuBLASLt (libgemm3_b200_cublaslt.so)"
    elif name in ("cutlass", "cudnn", "cute-dsl"):
        import flashinfer

        b, bsf = inp["b"], inp["b_sf"].reshape(n, k // 16)
        alpha = torch.ones((), device="cuda")

        def run():
            flashinfer.mm_fp4(inp["a"], b.T, inp["a_sf"].reshape(m, k // 16), bsf.T, alpha, out_dtype=out.dtype,
                              out=out, backend=name)

        keep = [b, bsf, alpha]
        with flashinfer.autotune(tune_mode=True):
            run()
        meta["autotuned"] = True
    else:
        raise ValueError(f"unsupported benchmark implementation: {name}")
    return run, out, meta, keep


def gpu_pids(uuid):
    """Compute processes on this GPU as nvidia-smi lists them (an empty list where the container
    hides other PID namespaces)."""
    try:
        return subprocess.check_output(
            ["nvidia-smi", "-i", uuid, "--query-compute-apps=pid", "--format=csv,noheader,nounits"], text=True,
            timeout=30,
        ).split()
    except (OSError, subprocess.SubprocessError) as exc:
        return [f"unavailable: {exc.__class__.__name__}"]


def run_compare(size, rounds, only, output, iters=50, out_dtype_name="float16"):
    import torch

    import gemm3_b200 as g3
    from gemm3_b200.testing import make_inputs

    out_dtype = getattr(torch, out_dtype_name)
    inp = make_inputs(size, size, size)
    cfg = g3.config_for(size, size, size)
    with g3.persisting_l2(cfg.persist_mb):
        refs = {
            dt: g3.gemm(inp["a"], inp["b"], inp["a_sf"], inp["b_sf"], out_dtype=dt, config=cfg)
            for dt in (torch.float16, torch.bfloat16)
        }
    # independent FP32 check at rows and columns spread across the whole output
    idx = torch.linspace(0, size - 1, 128, device="cuda").long()
    a = g3.dequantize_nvfp4(inp["a"][idx], inp["a_sf_linear"][idx])
    b = g3.dequantize_nvfp4(inp["b"][idx], inp["b_sf_linear"][idx])
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    sample_ref = a @ b.T
    torch.backends.cuda.matmul.allow_tf32 = prev
    reference_checks = {str(dt): accuracy(o[idx][:, idx], sample_ref) for dt, o in refs.items()}

    props = torch.cuda.get_device_properties(torch.cuda.current_device())
    uuid = "GPU-" + str(props.uuid).removeprefix("GPU-")
    expected = gpu_pids(uuid)

    def check_exclusive():
        actual = gpu_pids(uuid)
        if actual != expected:
            raise RuntimeError(f"GPU process set changed from {expected} to {actual}; discard this run")
        return actual

    data = dict(
        size=size, rounds=rounds, date=time.strftime("%Y-%m-%dT%H:%M:%SZ", time.gmtime()),
        gpu=torch.cuda.get_device_name(), gpu_uuid=uuid, torch=torch.__version__,
        timing=(f"CUDA events around one CUDA-graph replay per sample; cold L2 (flush of 2 x L2 before each); "
                f"1 ms cooldown; {iters} samples/round (CUPTI is not installed here)"),
        reference_checks=reference_checks, results={}, errors={}, gpu_checks=[],
        initial_compute_pids=expected,
        config=dict(tile=cfg.tile, cluster=cfg.cluster, fallback=cfg.fallback, persist_mb=cfg.persist_mb,
                    attrs=cfg.attr_dict()),
        source_sha256=source_hashes(),
    )
    output = Path(output)

    def save():
        data["loaded_libraries"] = sorted(
            {
                line.split()[-1]
                for line in Path("/proc/self/maps").read_text().splitlines()
                if any(x in line for x in ("libgemm3_b200", "libcublas", "libcudnn", "libcupti", "libnvrtc"))
            }
        )
        output.parent.mkdir(parents=True, exist_ok=True)
        output.write_text(json.dumps(data, indent=2) + "\n")

    runners = {}
    for name in only:
        check_exclusive()
        print(f"Preparing {name} at {size}", flush=True)
        try:
            run, out, meta, keep = adapter(name, inp, size, out_dtype)
            with g3.persisting_l2(cfg.persist_mb if name == "preset" else 0):
                run()
                torch.cuda.synchronize()
            meta.update(dtype=str(out.dtype), correctness=accuracy(out, refs[out.dtype]), samples_us=[])
            data["results"][name] = meta
            runners[name] = (run, keep)
            print(f"Ready {name}: {meta['correctness']}", flush=True)
        except Exception as exc:  # recorded, as the reference does, and the run goes on
            data["errors"][name] = repr(exc)
            print(f"FAILED {name}: {exc!r}", flush=True)
        save()
    names = list(runners)
    if not names:
        raise RuntimeError("no implementation passed validation")
    for rnd in range(rounds):
        data["gpu_checks"].append(dict(round=rnd + 1, compute_pids=check_exclusive()))
        for name in rotated_order(names, rnd):
            check_exclusive()
            run, _ = runners[name]
            with g3.persisting_l2(cfg.persist_mb if name == "preset" else 0):
                us = time_us(run, iters=iters)
            meta = data["results"][name]
            meta["samples_us"].append(us)
            meta["median_us"] = statistics.median(meta["samples_us"])
            meta["tflops"] = 2 * size**3 / meta["median_us"] / 1e6
            print(f"Round {rnd + 1} {name}: {us:.3f} us", flush=True)
            check_exclusive()
            save()
    return data


def summarize(paths):
    """Rows (size, implementation, median us, PF/s, bit_exact) from result files."""
    rows = []
    for path in paths:
        data = json.loads(Path(path).read_text())
        for name, meta in data.get("results", {}).items():
            if "median_us" in meta:
                rows.append(dict(size=data["size"], name=name, us=meta["median_us"],
                                 pflops=2 * data["size"] ** 3 / meta["median_us"] / 1e9,
                                 bit_exact=meta["correctness"]["bit_exact"], gpu=data.get("gpu", "")))
    order = {n: i for i, n in enumerate(LIBRARIES)}
    return sorted(rows, key=lambda r: (r["size"], order.get(r["name"], 99), r["name"]))


def markdown(rows):
    lines = ["| size | implementation | median µs | PF/s | bit-exact with gemm3_b200 |", "|---:|---|---:|---:|---|"]
    for r in rows:
        lines.append(f"| {r['size']}³ | {LABELS.get(r['name'], r['name'])} | {r['us']:.2f} | {r['pflops']:.2f} | "
                     f"{'yes' if r['bit_exact'] else 'no'} |")
    return "\n".join(lines) + "\n"


def svg(rows, width=720, bar_h=16, gap=6):
    """Horizontal bar chart of PF/s per size and implementation (the figures/plot.py throughput
    panel, drawn as plain SVG because no plotting library is installed here)."""
    from xml.sax.saxutils import escape

    colors = {"preset": "#8064A2", "cublaslt": "#6D9E9A", "cutlass": "#6D9E9A", "cudnn": "#6D9E9A",
              "cute-dsl": "#7D93AD"}
    peak = max((r["pflops"] for r in rows), default=1.0)
    left, right = 230, 70
    scale = (width - left - right) / peak
    y = 30
    parts = []
    for size in sorted({r["size"] for r in rows}):
        parts.append(f'<text x="8" y="{y + 12}" font-weight="bold">{size}³</text>')
        y += 20
        for r in (r for r in rows if r["size"] == size):
            w = max(1.0, r["pflops"] * scale)
            parts.append(f'<text x="8" y="{y + bar_h - 4}">{escape(LABELS.get(r["name"], r["name"]))}</text>')
            parts.append(f'<rect x="{left}" y="{y}" width="{w:.1f}" height="{bar_h}" '
                         f'fill="{colors.get(r["name"], "#999999")}"/>')
            parts.append(f'<text x="{left + w + 6:.1f}" y="{y + bar_h - 4}">{r["pflops"]:.2f}</text>')
            y += bar_h + gap
        y += 8
    head = (f'<svg xmlns="http://www.w3.org/2000/svg" width="{width}" height="{y + 10}" '
            f'font-family="DejaVu Sans, sans-serif" font-size="11">'
            f'<text x="8" y="16" font-size="12">NVFP4 GEMM throughput, PF/s (median of rounds)</text>')
    return head + "".join(parts) + "</svg>\n"


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    sub = ap.add_subparsers(dest="cmd", required=True)
    r = sub.add_parser("run")
    r.add_argument("--size", type=int, required=True)
    r.add_argument("--rounds", type=int, default=8)
    r.add_argument("--iters", type=int, default=50)
    r.add_argument("--only", default="preset,cublaslt")
    r.add_argument("--out-dtype", default="float16", choices=["float16", "bfloat16"])
    r.add_argument("--output", type=Path, required=True)
    sm = sub.add_parser("summary")
    sm.add_argument("results", nargs="+")
    sm.add_argument("--markdown", type=Path)
    sm.add_argument("--svg", type=Path)
    args = ap.parse_args(argv)
    if args.cmd == "run":
        run_compare(args.size, args.rounds, args.only.split(","), args.output, iters=args.iters,
                    out_dtype_name=args.out_dtype)
        return 0
    rows = summarize(args.results)
    table = markdown(rows)
    print(table, end="")
    if args.markdown:
        args.markdown.write_text(table)
    if args.svg:
        args.svg.write_text(svg(rows))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
