"""CPU: bench.py's workload arithmetic for the BASELINE configs (weak scaling by default, strong
scaling with --n-total, outlier injection flag), without a GPU."""

import sys

import pytest

import bench


def _args(monkeypatch, *argv):
    monkeypatch.setattr(sys, "argv", ["bench.py", *argv])
    return bench.parse()


def test_default_is_weak_scaling(monkeypatch):
    a = _args(monkeypatch, "--gpus", "8")
    assert bench.n_per_gpu(a) == 8192 and bench.scaling(a) == "weak"
    assert bench.workload_config(a)["workload"].startswith("NVFP4 GEMM 8192x65536x8192")


def test_config3_strong_scaling_with_outliers(monkeypatch):
    a = _args(monkeypatch, "--gpus", "8", "--size", "32768", "--n-total", "32768", "--outliers", "0.001")
    assert bench.n_per_gpu(a) == 4096 and bench.scaling(a) == "strong"
    cfg = bench.workload_config(a)
    assert cfg["n_per_gpu"] == 4096 and "32768x32768x32768" in cfg["workload"] and "0.001" in cfg["workload"]


def test_n_total_must_split_into_row_blocks(monkeypatch):
    with pytest.raises(SystemExit):
        _args(monkeypatch, "--gpus", "3", "--n-total", "1024")
