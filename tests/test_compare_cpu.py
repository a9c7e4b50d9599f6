"""CPU: the comparison harness's bookkeeping (gemm3_b200.compare): rotated round order, source
hashes, and the summary table and chart read from result files."""

import json
import xml.etree.ElementTree as ET

from gemm3_b200 import compare


def test_rotated_order_matches_the_reference_rule():
    names = ["preset", "cublaslt", "cutlass"]
    assert compare.rotated_order(names, 0) == ["preset", "cublaslt", "cutlass"]
    assert compare.rotated_order(names, 1) == ["preset", "cutlass", "cublaslt"]  # start 1, reversed
    assert compare.rotated_order(names, 2) == ["cutlass", "preset", "cublaslt"]
    assert compare.rotated_order(names, 3) == ["cutlass", "cublaslt", "preset"]  # start 0, reversed


def test_source_hashes_cover_kernels_and_headers():
    h = compare.source_hashes()
    assert any(k.endswith("csrc/gemm_pair_kernel.cuh") for k in h)
    assert any(k.endswith("include/nvfp4_gemm.h") for k in h)
    assert all(len(v) == 64 for v in h.values())


def test_summary_table_and_svg(tmp_path):
    for size, us in ((4096, 41.3), (8192, 218.5)):
        data = {"size": size, "gpu": "NVIDIA B200", "results": {
            "preset": {"median_us": us, "correctness": {"bit_exact": True}},
            "cublaslt": {"median_us": us * 0.9, "correctness": {"bit_exact": True}},
            "cutlass": {"samples_us": [], "correctness": {"bit_exact": False}},  # never timed: skipped
        }}
        (tmp_path / f"c{size}.json").write_text(json.dumps(data))
    rows = compare.summarize(sorted(str(p) for p in tmp_path.glob("*.json")))
    assert [(r["size"], r["name"]) for r in rows] == [(4096, "preset"), (4096, "cublaslt"), (8192, "preset"),
                                                       (8192, "cublaslt")]
    assert abs(rows[2]["pflops"] - 2 * 8192**3 / 218.5 / 1e9) < 1e-9
    md = compare.markdown(rows)
    assert "| 8192³ | gemm3_b200 (this package) | 218.50 |" in md
    root = ET.fromstring(compare.svg(rows))
    assert root.tag.endswith("svg") and len([e for e in root.iter() if e.tag.endswith("rect")]) == 4
