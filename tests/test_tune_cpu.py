"""CPU: every configuration gemm3_b200.tune times is one the GEMM accepts for that shape."""

import warnings

import pytest

from gemm3_b200 import api, tune


@pytest.mark.parametrize("size", [4096, 8192, 16384, 32768, 1024])
def test_tune_candidates_pass_host_validation(size):
    names = set()
    for name, cfg in tune.candidates(size):
        assert name not in names
        names.add(name)
        with warnings.catch_warnings():
            warnings.simplefilter("error")  # no fast_swz fallback: every band divides the M clusters
            attrs = api._effective_attrs(size, cfg)
        api._check_shape_guards(size, size, size, cfg, attrs)
    assert {"preset", "default", "tile (128, 256)"} <= names


def test_tune_markdown_table():
    rows = [dict(size=8192, config="preset", tile=[256, 256], cluster=[8, 2], attrs={"fast_swz": 2}, us=217.0,
                 pflops=5.07, bit_identical=True)]
    table = tune.markdown(rows)
    assert "| 8192 | preset | (256, 256) | fast_swz=2 | 217.0 | 5.07 | yes |" in table
