// Weight-streaming NVFP4 GEMM for skinny M (M <= 128) on sm_100a.
//
//   C[M,N] = alpha * A[M,K] . B[N,K]^T,  computed as  C^T[N,M] = B . A^T
//
// With few rows of A (the tokens of an LLM projection), the standard tiling wastes the tensor
// core's M dimension on absent rows and gives only N/256 tiles to 148 SMs. Here B, the weight,
// fills the MMA's M = 128 (one tile = 128 rows of B = 128 columns of C) and all rows of A form
// the MMA's N (A rows rounded up to 16). Every CTA reads the small A from L2 and streams its
// own rows of B from HBM once, so the kernel runs at the rate B leaves HBM. N/128 tiles spread
// over the persistent grid (224 for N = 28672).
//
// A stage covers K = 512: two 128-byte swizzle atoms of B (128 rows) and of A, plus eight
// 512-byte scale chunks of each operand. Stages fill the shared memory (5 at M <= 16, 3 at 128).
// Roles (9 warps):
//   warp 0      B producer: TMA loads of B (two 128-byte swizzle atoms of 128 rows) and bulk
//               copies of B's scale chunks;
//   warp 8      A producer: TMA loads of A and bulk copies of A's scales (from L2: every CTA
//               reads all of A). One thread issuing both operands took ~800 cycles per stage.
//               Both producers start as soon as the barriers are initialised; warp 1 allocates
//               TMEM meanwhile and hands it to warps 1-7 through named barrier 1, so the first
//               loads are not delayed by the allocation (about 1 us at kernel start);
//   warp 1      TMEM owner and MMA issuer: one wait per stage, then eight tcgen05.mma
//               (kind::mxf4nvf4, M=128, N=rows of A, K=64) into one of two accumulator buffers;
//   warps 2, 3  scale copies into TMEM (tcgen05.cp 32x128b.warpx4): warp 3 B's chunks, warp 2
//               A's, into one of two TMEM regions; each hands its region to the MMA thread with
//               a fence + arrive and frees the stage's shared memory with a commit. The MMA
//               thread thus issues only MMAs (every tcgen05 instruction costs its issuing thread
//               tens of cycles);
//   warps 4-7   epilogue: thread (quadrant q, lane l) holds column n = 128 t + 32 q + l of C for
//               every row m; x alpha in FP32, round to FP16/BF16, store C[m, n] (a warp writes
//               64 contiguous bytes per row m), also into peer GPUs' buffers when asked.
// Each output element is accumulated over k = 0, 64, 128, ... in one MMA chain, in the same
// order as the other kernels of this library.
//
// Programmatic dependent launch (p.pdl): 1 waits for the preceding kernel before any load;
// 2 streams B and its scales without waiting and loads A, its scales and alpha after the wait,
// so the weight stream starts while the kernel that produced A (an activation quantiser) is
// still running. Mode 2 requires that the preceding kernel does not write B.
#pragma once
#include "gemm_kernel.cuh"

namespace g3 {

constexpr int kStreamTileN = 128;   // B rows per tile (the MMA's M)
constexpr int kStreamMaxM = 128;    // A rows (the MMA's N): all of A in one tile
constexpr int kStreamKBlocks = 8;   // 64-element blocks per stage: K = 512
constexpr int kStreamKAtoms = kStreamKBlocks / kKBlocksPerTile;      // 128-byte swizzle atoms per row (2)
constexpr int kStreamAtomBytes = kStreamTileN * kTileKBytes;         // 16 KiB: 128 rows x 128 B
constexpr int kStreamBBytes = kStreamKAtoms * kStreamAtomBytes;      // 32 KiB of B per stage
constexpr int kStreamSfBytes = kStreamKBlocks * kSfChunk;            // 4 KiB of scales per operand
constexpr int kStreamMaxStages = 8;
constexpr int kStreamSfRegions = 2;
constexpr int kStreamAccCols = 128;                                  // one accumulator buffer
constexpr int kStreamSfCol = 2 * kStreamAccCols;                     // scale regions after both buffers
constexpr int kStreamSfColsPerRegion = 2 * 4 * kStreamKBlocks;       // B scales 32 + A scales 32
static_assert(kStreamSfCol + kStreamSfRegions * kStreamSfColsPerRegion <= kTmemCols, "stream TMEM");
constexpr int kStreamThreads = 288;
constexpr int kStreamSmemLimit = 232448;  // dynamic shared memory per CTA on sm_100

// Shared memory of one stage for MMA N = n_mma (A rows rounded up to 16): B atoms, A atoms, B
// scales, A scales. Every part starts on a 1024-byte boundary (swizzle atoms) or a 4 KiB one.
__host__ __device__ constexpr int stream_stage_bytes(int n_mma) {
  return kStreamBBytes + kStreamKAtoms * n_mma * kTileKBytes + 2 * kStreamSfBytes;
}
// full[S], empty[S], ready[S], acc_full[2], acc_empty[2], drain[3]; TMEM slot; abort flag
__host__ __device__ constexpr int stream_bar_bytes(int stages) { return (3 * stages + 7) * 8 + 8; }
__host__ __device__ constexpr int stream_stages(int n_mma) {
  return (kStreamSmemLimit - 1024 - stream_bar_bytes(kStreamMaxStages)) / stream_stage_bytes(n_mma) >
                 kStreamMaxStages
             ? kStreamMaxStages
             : (kStreamSmemLimit - 1024 - stream_bar_bytes(kStreamMaxStages)) / stream_stage_bytes(n_mma);
}
__host__ __device__ constexpr int stream_smem_bytes(int n_mma) {
  return stream_stages(n_mma) * stream_stage_bytes(n_mma) + stream_bar_bytes(stream_stages(n_mma)) + 1024;
}
static_assert(stream_stages(kStreamMaxM) >= 2, "stream kernel needs two stages at M = 128");
// A copy warp waits for completion (g - R) / S of empty[(g - R) % S] by parity; that barrier's
// next completion (iteration g - R + S) must lie after the copy warp's own iteration g, or the
// wait can miss a phase: R < S at every stage count.
static_assert(kStreamSfRegions < stream_stages(kStreamMaxM), "TMEM scale regions must be fewer than stages");
static_assert(stream_smem_bytes(16) <= kStreamSmemLimit && stream_smem_bytes(kStreamMaxM) <= kStreamSmemLimit,
              "stream kernel exceeds shared memory");

struct StreamParams {
  const uint8_t* sfa;  // A scales (swizzled); only row block 0 exists for M <= 128
  const uint8_t* sfb;  // B scales (swizzled)
  void* c;
  int64_t ldc, col0;  // output addressing, as in GemmParams
  int n_peer;
  void* peer[kMaxPeers];
  const float* alpha;
  int* status;
  int m, n;
  int n_mma;       // A rows rounded up to 16: the MMA's N
  int a_box_rows;  // A rows rounded up to 8: the TMA box height
  int sf_kblocks;  // K / 64
  int k_iters;     // stages per tile
  int num_tiles;   // ceil(N / 128)
  int stages;
  int stage_bytes;
  int pdl;
  int pol_b, pol_sfb;
};

// kOutView: C is a strided view (ldc, col0) and/or also stored into peer buffers (the fused
// gather); false compiles the contiguous [M, N] store alone.
template <bool kBF16, bool kOutView>
__global__ void __launch_bounds__(kStreamThreads, 1)
    nvfp4_gemm_stream_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                             const StreamParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int S = p.stages;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S * p.stage_bytes);
  uint64_t* empty = full + S;      // MMA commit + one commit per copy warp
  uint64_t* ready = empty + S;     // one arrive per copy warp: scales in TMEM, stage data landed
  uint64_t* acc_full = ready + S;  // [2]
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* drain = acc_empty + 2;  // [0] MMA, [1] B-scale copies, [2] A-scale copies
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 3);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  // stage layout
  const int off_a = kStreamBBytes;
  const int a_atom_bytes = p.n_mma * kTileKBytes;
  const int off_sfb = off_a + kStreamKAtoms * a_atom_bytes;
  const int off_sfa = off_sfb + kStreamSfBytes;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 2);   // one arrive.expect_tx from each producer
      mbar_init(&empty[s], 3);  // MMA commit + one commit per copy warp
      mbar_init(&ready[s], 2);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 4 * 32);
    }
    for (int d = 0; d < 3; ++d) mbar_init(&drain[d], 1);
    *abort_flag = 0;
    fence_mbarrier_init();
    prefetch_tmap(&tmap_b);
    prefetch_tmap(&tmap_a);
  }
  __syncthreads();  // barriers initialised; the producers start now, before TMEM is allocated

  uint32_t tmem = 0;
  if (warp >= 1 && warp <= 7) {
    // TMEM for the MMA, copy and epilogue warps only: allocated while the first loads fly.
    if (warp == 1) {
      tmem_alloc(tmem_slot, kTmemCols);
      tmem_relinquish();
    }
    tc_fence_before();
    asm volatile("bar.sync 1, %0;" ::"n"(7 * 32) : "memory");
    tc_fence_after();
    tmem = *tmem_slot;
  }

  if (warp == 0) {
    // ------------------------------------------------------------------ B producer (one thread)
    if (lane == 0) {
      const uint64_t pol_b = make_policy(p.pol_b);
      const uint64_t pol_sfb = make_policy(p.pol_sfb);
      if (p.pdl == 1) griddep_wait();  // mode 2: the weights do not depend on the preceding kernel
      uint32_t stage = 0, phase = 0, issued = 0, parity = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < p.num_tiles; t += gridDim.x) {
        for (int kt = 0; kt < p.k_iters; ++kt) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, p.status, kStatusTimeoutEmpty, abort_flag)) {
            ok = false;
            break;
          }
          const int nkb = min(kStreamKBlocks, p.sf_kblocks - kStreamKBlocks * kt);
          const uint32_t sf_bytes = static_cast<uint32_t>(nkb * kSfChunk);
          mbar_arrive_expect_tx(&full[stage], kStreamBBytes + sf_bytes);
          uint8_t* st = smem + stage * p.stage_bytes;
          const int x0 = kt * kStreamKAtoms * kTileKBytes;
#pragma unroll
          for (int h = 0; h < kStreamKAtoms; ++h)
            tma_load_2d(st + h * kStreamAtomBytes, &tmap_b, x0 + h * kTileKBytes, t * kStreamTileN, &full[stage],
                        pol_b);
          bulk_load(st + off_sfb,
                    p.sfb + (static_cast<size_t>(t) * p.sf_kblocks + static_cast<size_t>(kStreamKBlocks) * kt) * kSfChunk,
                    sf_bytes, &full[stage], pol_sfb);
          issued |= 1u << stage;
          parity = (parity & ~(1u << stage)) | (phase << stage);
          if (++stage == static_cast<uint32_t>(S)) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (ok) {
        // Tail: every stage released (MMA and copy commits arrived), so no tcgen05.commit
        // arrival is still in flight when the CTA exits.
        for (int s = 0; s < S; ++s) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, p.status, kStatusTimeoutEmpty, abort_flag)) break;
          if (++stage == static_cast<uint32_t>(S)) {
            stage = 0;
            phase ^= 1u;
          }
        }
      } else {
        // Unwind: let the copies already issued land before shared memory goes away.
        for (int s = 0; s < S; ++s)
          if (issued & (1u << s))
            mbar_wait(&full[s], (parity >> s) & 1u, p.status, kStatusTimeoutDrain, nullptr);
      }
    }
    __syncwarp();
  } else if (warp == 8) {
    // ------------------------------------------------------------------ A producer (one thread)
    // A (the few token rows), A's scales and alpha may come from the preceding kernel: with pdl
    // this thread waits for it before the first load.
    if (lane == 0) {
      if (p.pdl != 0) griddep_wait();
      const uint64_t pol_a = policy_evict_last();  // every CTA reads all of A
      const uint32_t a_bytes = static_cast<uint32_t>(kStreamKAtoms * p.a_box_rows * kTileKBytes);
      uint32_t stage = 0, phase = 0, issued = 0, parity = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < p.num_tiles; t += gridDim.x) {
        for (int kt = 0; kt < p.k_iters; ++kt) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, p.status, kStatusTimeoutEmpty, abort_flag)) {
            ok = false;
            break;
          }
          const int nkb = min(kStreamKBlocks, p.sf_kblocks - kStreamKBlocks * kt);
          const uint32_t sf_bytes = static_cast<uint32_t>(nkb * kSfChunk);
          mbar_arrive_expect_tx(&full[stage], a_bytes + sf_bytes);
          uint8_t* st = smem + stage * p.stage_bytes;
          const int x0 = kt * kStreamKAtoms * kTileKBytes;
#pragma unroll
          for (int h = 0; h < kStreamKAtoms; ++h)
            tma_load_2d(st + off_a + h * a_atom_bytes, &tmap_a, x0 + h * kTileKBytes, 0, &full[stage], pol_a);
          bulk_load(st + off_sfa, p.sfa + static_cast<size_t>(kStreamKBlocks) * kt * kSfChunk, sf_bytes, &full[stage],
                    pol_a);
          issued |= 1u << stage;
          parity = (parity & ~(1u << stage)) | (phase << stage);
          if (++stage == static_cast<uint32_t>(S)) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok) {
        for (int s = 0; s < S; ++s)
          if (issued & (1u << s))
            mbar_wait(&full[s], (parity >> s) & 1u, p.status, kStatusTimeoutDrain, nullptr);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer (one thread)
    if (lane == 0) {
      const uint32_t idesc = idesc_nvf4(kStreamTileN, p.n_mma);
      const uint32_t a_atom16 = static_cast<uint32_t>(a_atom_bytes >> 4);
      uint32_t stage = 0, phase = 0, region = 0;
      bool ok = true;
      int lt = 0;
      for (int t = blockIdx.x; ok && t < p.num_tiles; t += gridDim.x, ++lt) {
        const uint32_t buf = static_cast<uint32_t>(lt & 1);
        if (!mbar_wait(&acc_empty[buf], ((lt >> 1) & 1) ^ 1u, p.status, kStatusTimeoutAccEmpty, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t dacc = tmem + buf * kStreamAccCols;
        for (int kt = 0; kt < p.k_iters; ++kt) {
          if (!mbar_wait(&ready[stage], phase, p.status, kStatusTimeoutFull, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const int nkb = min(kStreamKBlocks, p.sf_kblocks - kStreamKBlocks * kt);
          const uint8_t* st = smem + stage * p.stage_bytes;
          // MMA A = the GEMM's B (weight rows), MMA B = the GEMM's A (token rows)
          const uint64_t dw = sdesc_kmajor_sw128(smem_u32(st));
          const uint64_t dx = sdesc_kmajor_sw128(smem_u32(st + off_a));
          const uint32_t tsw = tmem + kStreamSfCol + region * kStreamSfColsPerRegion;
          const uint32_t tsx = tsw + 4 * kStreamKBlocks;
          // block j: swizzle atom j / 4, 32-byte K step j % 4 inside it (descriptor units of 16 B)
          if (nkb == kStreamKBlocks) {
#pragma unroll
            for (int j = 0; j < kStreamKBlocks; ++j)
              tc_mma_nvf4(dacc, dw + (j >> 2) * (kStreamAtomBytes >> 4) + 2 * (j & 3),
                          dx + (j >> 2) * a_atom16 + 2 * (j & 3), idesc, tsw + 4 * j, tsx + 4 * j,
                          (kt | j) != 0 ? 1u : 0u);
          } else {
            for (int j = 0; j < nkb; ++j)
              tc_mma_nvf4(dacc, dw + (j >> 2) * (kStreamAtomBytes >> 4) + 2 * (j & 3),
                          dx + (j >> 2) * a_atom16 + 2 * (j & 3), idesc, tsw + 4 * j, tsx + 4 * j,
                          (kt | j) != 0 ? 1u : 0u);
          }
          tc_commit(&empty[stage]);
          if (++stage == static_cast<uint32_t>(S)) {
            stage = 0;
            phase ^= 1u;
          }
          if (++region == kStreamSfRegions) region = 0;
        }
        if (!ok) break;
        tc_commit(&acc_full[buf]);
      }
      if (!ok) {
        tc_commit(&drain[0]);
        mbar_wait(&drain[0], 0, p.status, kStatusTimeoutDrain, nullptr);
      }
    }
    __syncwarp();
  } else if (warp == 2 || warp == 3) {
    // ------------------------------------------------------------------ scale copies
    // Iteration g lands in TMEM region g % R once the MMAs of iteration g - R, the last readers
    // of that region, have completed: completion (g - R) / S of empty[(g - R) % S].
    if (lane == 0) {
      const bool is_w = warp == 3;
      const int src_off = is_w ? off_sfb : off_sfa;
      const uint32_t col_off = is_w ? 0u : 4u * kStreamKBlocks;
      uint32_t stage = 0, phase = 0, region = 0, lag_stage = 0, lag_phase = 0;
      int it = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < p.num_tiles; t += gridDim.x) {
        for (int kt = 0; kt < p.k_iters; ++kt, ++it) {
          if (!mbar_wait(&full[stage], phase, p.status, kStatusTimeoutFull, abort_flag)) {
            ok = false;
            break;
          }
          if (it >= kStreamSfRegions) {
            if (!mbar_wait(&empty[lag_stage], lag_phase, p.status, kStatusTimeoutEmpty, abort_flag)) {
              ok = false;
              break;
            }
            if (++lag_stage == static_cast<uint32_t>(S)) {
              lag_stage = 0;
              lag_phase ^= 1u;
            }
          }
          tc_fence_after();
          const int nkb = min(kStreamKBlocks, p.sf_kblocks - kStreamKBlocks * kt);
          const uint64_t dsrc = sdesc_sf_chunk(smem_u32(smem + stage * p.stage_bytes + src_off));
          const uint32_t dst = tmem + kStreamSfCol + region * kStreamSfColsPerRegion + col_off;
          if (nkb == kStreamKBlocks) {
#pragma unroll
            for (int j = 0; j < kStreamKBlocks; ++j) tc_cp_32x128b_warpx4(dst + 4 * j, dsrc + 32 * j);
          } else {
            for (int j = 0; j < nkb; ++j) tc_cp_32x128b_warpx4(dst + 4 * j, dsrc + 32 * j);
          }
          tc_fence_before();
          mbar_arrive(&ready[stage]);
          tc_commit(&empty[stage]);
          if (++stage == static_cast<uint32_t>(S)) {
            stage = 0;
            phase ^= 1u;
          }
          if (++region == kStreamSfRegions) region = 0;
        }
      }
      if (!ok) {
        const int role = is_w ? 1 : 2;
        tc_commit(&drain[role]);
        mbar_wait(&drain[role], 0, p.status, kStatusTimeoutDrain, nullptr);
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------------ epilogue (warps 4-7)
    const int quad = warp & 3;
    const uint32_t lane_base = static_cast<uint32_t>(quad * 32) << 16;
    if (p.pdl != 0) griddep_wait();  // alpha may come from the preceding kernel
    const float alpha = *p.alpha;
    int lt = 0;
    for (int t = blockIdx.x; t < p.num_tiles; t += gridDim.x, ++lt) {
      const uint32_t buf = static_cast<uint32_t>(lt & 1);
      if (!mbar_wait(&acc_full[buf], (lt >> 1) & 1, p.status, kStatusTimeoutAccFull, abort_flag)) break;
      tc_fence_after();
      const int n_idx = t * kStreamTileN + quad * 32 + lane;
      const bool valid = n_idx < p.n;
      for (int ch = 0; ch < p.n_mma; ch += 32) {
        uint32_t r[32];
        const uint32_t taddr = tmem + lane_base + buf * kStreamAccCols + static_cast<uint32_t>(ch);
        if (p.n_mma - ch >= 32)
          tmem_ld_32x32b_x32(taddr, r);
        else
          tmem_ld_32x32b_x16(taddr, r);
        tmem_ld_wait();
        const int rows = min(32, p.m - ch);
        if (valid && !kOutView) {
          // contiguous [M, N] output, no peers: C[m, n] = col[m * N]
          uint16_t* col = static_cast<uint16_t*>(p.c) + n_idx;
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            if (i < rows) {
              const float v = __fmul_rn(__uint_as_float(r[i]), alpha);
              uint16_t bits;
              if constexpr (kBF16)
                bits = __bfloat16_as_ushort(__float2bfloat16_rn(v));
              else
                bits = __half_as_ushort(__float2half_rn(v));
              col[static_cast<size_t>(ch + i) * p.n] = bits;
            }
          }
        } else if (valid && kOutView) {
          // strided view and/or the fused gather into the peers' buffers
          const size_t base = static_cast<size_t>(ch) * p.ldc + p.col0 + n_idx;
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            if (i < rows) {
              const float v = __fmul_rn(__uint_as_float(r[i]), alpha);
              uint16_t bits;
              if constexpr (kBF16)
                bits = __bfloat16_as_ushort(__float2bfloat16_rn(v));
              else
                bits = __half_as_ushort(__float2half_rn(v));
              const size_t e = base + static_cast<size_t>(i) * p.ldc;
              static_cast<uint16_t*>(p.c)[e] = bits;
              for (int d = 0; d < p.n_peer; ++d) static_cast<uint16_t*>(p.peer[d])[e] = bits;
            }
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&acc_empty[buf]);
    }
  }

  // Peer stores are visible to the other GPUs before this grid is seen as complete.
  if (kOutView && p.n_peer > 0) __threadfence_system();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

}  // namespace g3
