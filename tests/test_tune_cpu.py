"""CPU: every configuration gemm3_b200.tune times is one the GEMM accepts for that shape."""

import warnings

import pytest

from gemm3_b200 import api, tune


@pytest.mark.parametrize("shape", [(4096,) * 3, (8192,) * 3, (16384,) * 3, (32768,) * 3, (1024,) * 3,
                                   (32768, 4096, 32768), (8192, 28672, 8192), (1024, 28672, 8192)])
def test_tune_candidates_pass_host_validation(shape):
    m, n, k = shape
    names = set()
    for name, cfg in tune.candidates(m, n, k):
        assert name not in names
        names.add(name)
        with warnings.catch_warnings():
            warnings.simplefilter("error")  # no fast_swz fallback: every band divides the M clusters
            attrs = api._effective_attrs(m, cfg)
        api._check_shape_guards(m, n, k, cfg, attrs)
    assert {"preset", "default", "tile (128, 256)"} <= names
    assert any(cfg.persist_mb > 0 for _, cfg in tune.candidates(m, n, k))


def test_tune_markdown_table():
    rows = [dict(size=8192, config="preset", tile=[256, 256], cluster=[8, 2], attrs={"fast_swz": 2}, persist_mb=0,
                 us=217.0, pflops=5.07, bit_identical=True)]
    table = tune.markdown(rows)
    assert "| 8192 | preset | (256, 256) | fast_swz=2 | 0 | 217.0 | 5.07 | yes |" in table
