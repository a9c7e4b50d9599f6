"""GPU: the column-parallel GEMM across 2 GPUs with NCCL (gemm3_b200.dist).

Each rank quantises its block of B with B's global scale (all-reduced amax) and computes its
column block of C. Checked against one GPU doing the whole GEMM: the shard's codes and scales
equal the matching slice of the whole tensor quantised, the column blocks are bit-identical (the
same kernel with the same accumulation order per element), and the gathered C equals the whole
C. Needs at least two GPUs; on a one-GPU box it is skipped.
"""

import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _nccl_worker(rank, world, port, m, n, k, result_dir):
    import datetime

    import torch.distributed as dist

    import gemm3_b200 as g3
    from gemm3_b200 import dist as g3dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    try:
        g = torch.Generator(device=dev).manual_seed(5)
        a = torch.randn(m, k, device=dev, generator=g).to(torch.bfloat16)
        b_whole = torch.randn(n, k, device=dev, generator=g).to(torch.bfloat16)  # same on every rank
        b_whole[7, 3] = 40.0  # B's amax sits in rank 0's rows only: rank 1 needs the all-reduce
        start, stop = g3dist.shard_bounds(n, world, rank)
        b_local = b_whole[start:stop].contiguous()
        aq, asf, _, gsa = g3.quantize_nvfp4_global(a)
        bq_whole, bsf_whole, _, gsb_whole = g3.quantize_nvfp4_global(b_whole)
        bq, bsf, _, gsb = g3dist.quantize_shard_global(b_local)
        want_q, want_sf = g3dist.shard_quantized(bq_whole, bsf_whole, world, rank)
        ok = torch.equal(gsb.view(torch.int32), gsb_whole.view(torch.int32))
        ok = ok and torch.equal(bq, want_q) and torch.equal(bsf, want_sf)
        alpha = (1.0 / (gsa * gsb)).reshape(1)
        c_local = g3dist.gemm_column_parallel(aq, bq, asf, bsf, alpha=alpha, out_dtype=torch.bfloat16)
        c_whole = g3.gemm(aq, bq_whole, asf, bsf_whole, alpha=alpha, out_dtype=torch.bfloat16)
        ok = ok and torch.equal(c_local, c_whole[:, start:stop])
        c_gathered = g3dist.all_gather_columns(c_local)
        ok = ok and torch.equal(c_gathered, c_whole)
        ok = ok and g3.device_status() == 0
        torch.cuda.synchronize()
        with open(os.path.join(result_dir, f"rank{rank}"), "w") as f:
            f.write("ok" if ok else "mismatch")
    finally:
        dist.destroy_process_group()


def test_column_parallel_gemm_two_gpus(cuda_ext, tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp

    world = 2
    mp.spawn(_nccl_worker, args=(world, _free_port(), 384, 1024, 512, str(tmp_path)), nprocs=world, join=True)
    for r in range(world):
        assert (tmp_path / f"rank{r}").read_text() == "ok", r


def _gather_worker(rank, world, port, m, n, k, result_dir):
    import datetime

    import torch.distributed as dist

    import gemm3_b200 as g3
    from gemm3_b200 import dist as g3dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    gather = None
    try:
        g = torch.Generator(device=dev).manual_seed(9)
        a = torch.randn(m, k, device=dev, generator=g).to(torch.bfloat16)
        b_whole = torch.randn(n, k, device=dev, generator=g).to(torch.bfloat16)
        start, stop = g3dist.shard_bounds(n, world, rank)
        aq, asf, _, gsa = g3.quantize_nvfp4_global(a)
        bq_whole, bsf_whole, _, gsb = g3.quantize_nvfp4_global(b_whole)
        bq, bsf = g3dist.shard_quantized(bq_whole, bsf_whole, world, rank)
        gather = g3dist.PeerGather(m, n, dtype=torch.bfloat16)
        ok = True
        for scale in (1.0, 0.5):  # two calls in a row into the same buffers
            alpha = (scale / (gsa * gsb)).reshape(1)
            gather.full.fill_(float("nan"))
            gather.barrier()  # every rank's buffer reset before any rank writes into it
            full = g3dist.gemm_column_parallel_gather(aq, bq, asf, bsf, gather, alpha=alpha)
            want = g3.gemm(aq, bq_whole, asf, bsf_whole, alpha=alpha, out_dtype=torch.bfloat16)
            torch.cuda.synchronize()
            ok = ok and torch.equal(full, want)
        ok = ok and g3.device_status() == 0
        with open(os.path.join(result_dir, f"rank{rank}"), "w") as f:
            f.write("ok" if ok else "mismatch")
    finally:
        if gather is not None:
            gather.barrier()
            torch.cuda.synchronize()
            gather.close()
            dist.barrier()
        dist.destroy_process_group()


def test_fused_gather_two_gpus(cuda_ext, tmp_path):
    """The gather fused into the GEMM epilogue (peer stores over NVLink into every rank's full-C
    buffer): after the barrier, each rank's buffer equals the one-GPU GEMM bit for bit."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp

    world = 2
    # M = 320: the CTA-pair kernel; M = 64: the weight-streaming kernel (skinny-M preset)
    for m in (320, 64):
        mp.spawn(_gather_worker, args=(world, _free_port(), m, 1536, 1024, str(tmp_path)), nprocs=world, join=True)
        for r in range(world):
            assert (tmp_path / f"rank{r}").read_text() == "ok", (m, r)
