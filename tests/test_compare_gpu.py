"""GPU: the comparison harness end to end on a small size: reference checks, validation of
cuBLASLt against this package's output (bit-identical), rotated timed rounds and the JSON record."""

import json

import pytest

pytestmark = pytest.mark.gpu


def test_compare_run_small(cuda_ext, tmp_path):
    from gemm3_b200 import compare

    out = tmp_path / "compare-1024.json"
    data = compare.run_compare(1024, 2, ["preset", "cublaslt"], out, iters=5)
    saved = json.loads(out.read_text())
    assert saved["size"] == 1024 and len(saved["gpu_checks"]) == 2
    for dt in ("torch.float16", "torch.bfloat16"):
        assert saved["reference_checks"][dt]["finite"]
    assert not saved["errors"], saved["errors"]
    for name in ("preset", "cublaslt"):
        r = saved["results"][name]
        assert len(r["samples_us"]) == 2 and r["median_us"] > 0
    assert saved["results"]["cublaslt"]["correctness"]["bit_exact"]
    assert saved["results"]["preset"]["correctness"]["bit_exact"]
    assert any("libgemm3_b200" in lib for lib in saved["loaded_libraries"])
    assert data["source_sha256"] == saved["source_sha256"]
