"""Column-parallel NVFP4 GEMM, one process per GPU (torch.distributed).

C = alpha * dequant(A) @ dequant(B).T is split along N. Every rank holds all of A (and its scales)
and a block of N / g rows of B; rank r computes columns [r * N / g, (r + 1) * N / g) of C. The
GEMM itself exchanges nothing, so the work scales weakly with the rank count. Only two steps use
the process group:

- B's per-tensor global scale must be one value on every rank. The amax of each rank's rows is
  reduced with MAX before quantisation, so each rank's codes and scales equal the matching rows
  of B quantised whole (quantize_shard_global).
- Gathering C is optional. NCCL's all-gather of the [M, N / g] shards lays them out as
  [g][M][N / g]; a copy then rearranges that into row-major [M, N] (all_gather_columns). Or the
  gather is fused into the GEMM: PeerGather maps every rank's full [M, N] buffer into every
  other rank (CUDA IPC) and gemm_column_parallel_gather's epilogue stores each tile into all of
  them over NVLink, already row-major, followed by a one-element all-reduce as the barrier.

Nothing here depends on the backend: NCCL with CUDA tensors in production, gloo with CPU tensors
for the host-side logic in tests. The reference package is single-GPU; this module carries its
GEMM (nvfp4_gemm_cute/api.py:152-220) across the GPUs of one node.
"""

import ctypes

import torch
import torch.distributed as dist

from . import _lib
from .api import _check_shape_guards, _effective_attrs, _launch_config, _out_code, _status_word, gemm
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


class PeerGather:
    """Every rank's full row-major [M, N] output buffer, mapped into every other rank of the group.

    Each rank allocates `full` on its current GPU, exports it with CUDA IPC (nvfp4_ipc_get_handle),
    the handles are all-gathered through the process group and every rank opens the others'
    (nvfp4_ipc_open). `ptrs` lists this rank's buffer first, then the peers' in rank order: the
    destinations of gemm_column_parallel_gather. close() releases the mappings; call it on every
    rank before the buffers are freed. Legacy IPC mappings, no NVLink multicast objects.
    """

    def __init__(self, m, n, dtype=torch.float16, group=None):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.m, self.n, self.dtype = m, n, dtype
        dev = torch.device("cuda", torch.cuda.current_device())
        self.full = torch.empty(m, n, dtype=dtype, device=dev)
        L = _lib.lib()
        handle = (ctypes.c_uint8 * _lib.IPC_HANDLE_BYTES)()
        off = ctypes.c_int64(0)
        _lib.check(L.nvfp4_ipc_get_handle(self.full.data_ptr(), handle, ctypes.byref(off)), "nvfp4_ipc_get_handle")
        mine = torch.zeros(_lib.IPC_HANDLE_BYTES + 8, dtype=torch.uint8)
        mine[: _lib.IPC_HANDLE_BYTES] = torch.tensor(list(bytes(handle)), dtype=torch.uint8)
        mine[_lib.IPC_HANDLE_BYTES :] = torch.tensor(list(off.value.to_bytes(8, "little")), dtype=torch.uint8)
        table = torch.empty(self.world * mine.numel(), dtype=torch.uint8, device=dev)
        dist.all_gather_into_tensor(table, mine.to(dev), group=group)
        table = table.view(self.world, -1).cpu()
        self._opened = []
        ptrs = [self.full.data_ptr()]
        for r in range(self.world):
            if r == self.rank:
                continue
            h = (ctypes.c_uint8 * _lib.IPC_HANDLE_BYTES)(*table[r, : _lib.IPC_HANDLE_BYTES].tolist())
            o = int.from_bytes(bytes(table[r, _lib.IPC_HANDLE_BYTES :].tolist()), "little")
            p = ctypes.c_void_p(0)
            _lib.check(L.nvfp4_ipc_open(h, o, ctypes.byref(p)), "nvfp4_ipc_open")
            self._opened.append((p.value, o))
            ptrs.append(p.value)
        self.ptrs = ptrs
        self._dst = (ctypes.c_void_p * len(ptrs))(*ptrs)
        self._flag = torch.zeros(1, dtype=torch.float32, device=dev)

    def barrier(self):
        """Order every later reader on this rank's stream after every rank's gather GEMM."""
        dist.all_reduce(self._flag, group=self.group)

    def close(self):
        L = _lib.lib()
        for p, o in self._opened:
            L.nvfp4_ipc_close(p, o)
        self._opened = []


def gemm_column_parallel_gather(a, b_shard, a_sf, b_sf_shard, gather, alpha=None, out_dtype=None, config=None,
                                barrier=True):
    """This rank's block of C, written straight into every rank's full buffer (gather.full).

    Rank r's N/g columns go to columns [r * N/g, (r + 1) * N/g) of every buffer in gather.ptrs
    (nvfp4_gemm_run_gather). With barrier=True the call ends with gather.barrier(), after which
    gather.full on this rank holds all of C. Same operands and validation as gemm.
    """
    m, kp = a.shape
    n_local, k = b_shard.shape[0], kp * 2
    out_dtype = gather.dtype if out_dtype is None else out_dtype
    if out_dtype != gather.dtype:
        raise ValueError(f"out_dtype {out_dtype} differs from the gather buffers' {gather.dtype}")
    if m != gather.m or n_local * gather.world != gather.n:
        raise ValueError(f"[{m}, {n_local}] blocks from {gather.world} ranks do not make [{gather.m}, {gather.n}]")
    if b_shard.shape[1] != kp:
        raise ValueError(f"K mismatch: a is [{m}, {kp}], b is [{n_local}, {b_shard.shape[1]}]")
    if n_local % 64 or k % 64:
        raise ValueError(f"N and K must be multiples of 64 (got N={n_local}, K={k})")
    cfg = config or config_for(m, n_local, k)
    attrs = _effective_attrs(m, cfg)
    _check_shape_guards(m, n_local, k, cfg, attrs)
    ccfg = _launch_config(m, k, cfg, attrs, 0)
    dev = a.device
    if alpha is None:
        alpha = torch.ones(1, dtype=torch.float32, device=dev)
    alpha = alpha.reshape(1).to(device=dev, dtype=torch.float32)
    status = _status_word(dev)
    L = _lib.lib()
    with torch.cuda.device(dev):
        rc = L.nvfp4_gemm_run_gather(
            a.data_ptr(), b_shard.data_ptr(), a_sf.data_ptr(), b_sf_shard.data_ptr(), gather._dst, len(gather.ptrs),
            gather.n, gather.rank * n_local, alpha.data_ptr(), m, n_local, k, _out_code(out_dtype),
            ctypes.byref(ccfg), status.data_ptr(), torch.cuda.current_stream(dev).cuda_stream,
        )
    _lib.check(rc, "nvfp4_gemm_run_gather")
    if barrier:
        gather.barrier()
    return gather.full
