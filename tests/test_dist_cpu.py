"""CPU: the host-side logic of the column-parallel GEMM (gemm3_b200.dist) with gloo ranks.

Sharding B: a block-aligned row range of a quantised B is a contiguous slice of its packed codes
and swizzled scales, and equals quantising those rows alone with the same global scale (checked
with the CPU oracle). Collectives: the all-reduced amax and the all-gather + relayout of C, run as
two gloo processes on this host.
"""

import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from gemm3_b200 import dist as g3dist
from oracle import oracle


def test_shard_bounds():
    assert g3dist.shard_bounds(1024, 2, 0) == (0, 512)
    assert g3dist.shard_bounds(1024, 2, 1) == (512, 1024)
    assert g3dist.shard_bounds(32768, 8, 7) == (28672, 32768)
    with pytest.raises(ValueError, match="whole 128-row blocks"):
        g3dist.shard_bounds(1024 + 64, 2, 0)
    with pytest.raises(ValueError):
        g3dist.shard_bounds(1024, 2, 2)


@pytest.mark.parametrize("world", [2, 4])
def test_shard_of_quantized_b_equals_quantized_rows(world):
    rng = np.random.default_rng(11)
    n, k = 1024, 320  # K with a partial 4-column scale group (20 scale columns)
    b = rng.standard_normal((n, k)).astype(np.float32)
    gs = float(np.float32(2688.0) / np.abs(b).max())
    packed, swz, _ = oracle.quantize(b, gs, div_mode=1)
    packed_t, swz_t = torch.from_numpy(packed), torch.from_numpy(swz)
    for rank in range(world):
        p_r, s_r = g3dist.shard_quantized(packed_t, swz_t, world, rank)
        start, stop = g3dist.shard_bounds(n, world, rank)
        want_p, want_s, _ = oracle.quantize(b[start:stop], gs, div_mode=1)
        np.testing.assert_array_equal(p_r.numpy(), want_p)
        np.testing.assert_array_equal(s_r.numpy(), want_s)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _gloo_worker(rank, world, port, m, n_local):
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        # C blocks: rank r holds columns [r * n_local, (r + 1) * n_local) of a known matrix
        full = torch.arange(m * world * n_local, dtype=torch.float32).reshape(m, world * n_local)
        c_shard = full[:, rank * n_local : (rank + 1) * n_local].contiguous()
        got = g3dist.all_gather_columns(c_shard)
        assert torch.equal(got, full), "all-gather relayout differs from the full matrix"
        # global amax: each rank holds rows with a different maximum
        x = torch.full((4, 16), -0.5 - rank, dtype=torch.float32)
        amax = g3dist.global_amax(x)
        assert amax.item() == 0.5 + (world - 1), amax
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2])
def test_gloo_all_gather_columns_and_global_amax(world):
    mp.spawn(_gloo_worker, args=(world, _free_port(), 6, 5), nprocs=world, join=True)
