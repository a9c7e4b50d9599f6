"""Column-parallel NVFP4 GEMM, one process per GPU (torch.distributed).

C = alpha * dequant(A) @ dequant(B).T is split along N. Every rank holds all of A (and its scales)
and a block of N / g rows of B; rank r computes columns [r * N / g, (r + 1) * N / g) of C. The
GEMM itself exchanges nothing, so the work scales weakly with the rank count. Only two steps use
the process group:

- B's per-tensor global scale must be one value on every rank. The amax of each rank's rows is
  reduced with MAX before quantisation, so each rank's codes and scales equal the matching rows
  of B quantised whole (quantize_shard_global).
- Gathering C is optional. NCCL's all-gather of the [M, N / g] shards lays them out as
  [g][M][N / g]; a copy then rearranges that into row-major [M, N] (all_gather_columns).

Nothing here depends on the backend: NCCL with CUDA tensors in production, gloo with CPU tensors
for the host-side logic in tests. The reference package is single-GPU; this module carries its
GEMM (nvfp4_gemm_cute/api.py:152-220) across the GPUs of one node.
"""

import torch
import torch.distributed as dist

from .api import gemm
from .presets import config_for
from .quant import SF_VEC, _run_quantize, tensor_amax

ROW_BLOCK = 128  # rows per block of the swizzled scale layout


def shard_bounds(n: int, world: int, rank: int):
    """[start, stop) of the B rows (C columns) that `rank` owns.

    N must split into `world` shards of whole 128-row blocks (N % (world * 128) == 0), so that
    every shard's scales are a contiguous slice of the swizzled layout.
    """
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} is not in a group of {world}")
    if n % (world * ROW_BLOCK):
        raise ValueError(f"N={n} does not split into {world} shards of whole {ROW_BLOCK}-row blocks")
    per = n // world
    return rank * per, (rank + 1) * per


def sf_block_bytes(k: int) -> int:
    """Bytes of one 128-row block of the swizzled scale layout for reduction length K."""
    return ROW_BLOCK * (-(-(k // SF_VEC) // 4)) * 4


def shard_quantized(packed, sf_swizzled, world: int, rank: int):
    """This rank's rows of a quantised B: (packed [N/g, K/2], swizzled scales), as views.

    The swizzled layout stores the 128-row blocks one after another, each sf_block_bytes(K)
    long, so a block-aligned row range is one contiguous slice of it.
    """
    n, half_k = packed.shape
    start, stop = shard_bounds(n, world, rank)
    blk = sf_block_bytes(2 * half_k)
    sf = sf_swizzled.reshape(-1)
    if sf.numel() != (n // ROW_BLOCK) * blk:
        raise ValueError(f"scale tensor has {sf.numel()} bytes, expected {(n // ROW_BLOCK) * blk}")
    return packed[start:stop], sf[start // ROW_BLOCK * blk : stop // ROW_BLOCK * blk]


def global_amax(x_shard, group=None):
    """max |x| over every rank's shard, as a one-element float32 tensor on x_shard's device.

    The local amax (a CUDA kernel for CUDA tensors) is all-reduced with MAX. A NaN in any
    shard is carried only as far as the backend's MAX carries NaN.
    """
    if x_shard.device.type == "cuda":
        amax = tensor_amax(x_shard)
    else:
        amax = x_shard.float().abs().amax().reshape(1)
    dist.all_reduce(amax, op=dist.ReduceOp.MAX, group=group)
    return amax


def quantize_shard_global(x_shard, group=None):
    """Quantise this rank's rows of a tensor with the tensor's global encode scale
    gs = 2688 / amax(all ranks), bit-identical to the same rows of quantize_nvfp4_global on the
    whole tensor. Needs a CUDA tensor.

    Returns:
        (packed, sf_swizzled, sf_linear, global_scale) as quantize_nvfp4_global.
    """
    if x_shard.device.type != "cuda":
        raise ValueError("quantize_shard_global needs a CUDA tensor")
    amax = global_amax(x_shard, group)
    return _run_quantize(x_shard, 0.0, amax, 2, 0, want_gs=True)


def gemm_column_parallel(a, b_shard, a_sf, b_sf_shard, alpha=None, out=None, out_dtype=torch.float16, config=None):
    """This rank's block of C, [M, N / g] = alpha * dequant(A) @ dequant(B_shard).T.

    A local call of gemm(); the launch configuration is chosen for the local shape unless
    `config` is given.
    """
    m, half_k = a.shape
    cfg = config if config is not None else config_for(m, b_shard.shape[0], 2 * half_k)
    return gemm(a, b_shard, a_sf, b_sf_shard, alpha=alpha, out=out, out_dtype=out_dtype, config=cfg)


def all_gather_columns(c_shard, group=None, out=None, gathered=None):
    """The full C [M, N] from every rank's [M, N / g] block.

    An all-gather into [g * M, N / g] (the shards stacked, the collective's own layout), then one
    copy that rearranges it into row-major [M, N]. `out` and `gathered` may be passed in to reuse
    buffers.
    """
    world = dist.get_world_size(group)
    m, n_local = c_shard.shape
    if gathered is None:
        gathered = torch.empty((world * m, n_local), dtype=c_shard.dtype, device=c_shard.device)
    dist.all_gather_into_tensor(gathered, c_shard.contiguous(), group=group)
    if out is None:
        out = torch.empty((m, world * n_local), dtype=c_shard.dtype, device=c_shard.device)
    out.view(m, world, n_local).copy_(gathered.view(world, m, n_local).permute(1, 0, 2))
    return out
