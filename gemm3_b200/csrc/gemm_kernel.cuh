// Persistent, warp-specialised NVFP4 block-scaled GEMM for sm_100a.
//
//   C[M,N] = alpha * sum_k deq(A)[m,k] * deq(B)[n,k]       (A: [M,K/2] u8, B: [N,K/2] u8)
//
// One CTA per SM computes 128x256 output tiles in a static persistent schedule:
//   warp 0      TMA producer: A (128 rows x 128 B) and B (256 rows x 128 B) tiles with the
//               128-byte swizzle, plus the matching swizzled scale chunks as plain bulk copies,
//               into a 4-stage shared-memory ring;
//   warp 1      TMEM owner and MMA issuer: per k-tile (256 FP4 = 128 B per row) it copies the
//               scale chunks into TMEM (tcgen05.cp 32x128b.warpx4) and issues up to four
//               tcgen05.mma kind::mxf4nvf4 block16 instructions (M=128, N=256, K=64);
//   warps 2-5   epilogue: TMEM -> registers (tcgen05.ld 32x32b.x32), x alpha in FP32, round to
//               FP16/BF16, release the accumulator, then 256-bit stores of each thread's row.
// Each output element is accumulated in the same order (k = 0, 64, 128, ...) whatever the
// raster, band or cache settings, so the result bits do not depend on the launch configuration.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "ptx.cuh"

namespace g3 {

constexpr int kTileM = 128;
constexpr int kTileN = 256;
constexpr int kTileKBytes = 128;  // 256 FP4 elements per row per k-tile
constexpr int kKBlocksPerTile = 4;  // 64-element scale blocks (one MMA each) per k-tile
constexpr int kStages = 4;
constexpr int kABytes = kTileM * kTileKBytes;   // 16 KiB
constexpr int kBBytes = kTileN * kTileKBytes;   // 32 KiB
constexpr int kSfChunk = 512;                   // 128 rows x 4 scales
constexpr int kSfaBytes = kKBlocksPerTile * kSfChunk;       // 2 KiB
constexpr int kSfbBytes = 2 * kKBlocksPerTile * kSfChunk;   // 4 KiB
constexpr int kTmemCols = 512;
constexpr int kAccCol = 0;
// Scale factors get one TMEM region per shared-memory stage, so the copies for k-tile t+1 never
// overwrite columns that the MMAs of k-tile t are still reading (that hazard drains the tensor
// pipe once per k-tile). Per stage: SFA 4 columns per 64-element block, SFB 8 (two 128-row halves).
constexpr int kSfColsPerStage = 4 * kKBlocksPerTile + 8 * kKBlocksPerTile;  // 48
constexpr int kSfaCol = 256;
constexpr int kSfbCol = kSfaCol + 4 * kKBlocksPerTile;
static_assert(kSfaCol + kStages * kSfColsPerStage <= kTmemCols, "scale factors do not fit in TMEM");
constexpr int kGemmThreads = 192;

constexpr int kOffA = 0;
constexpr int kOffB = kOffA + kStages * kABytes;
constexpr int kOffSfa = kOffB + kStages * kBBytes;
constexpr int kOffSfb = kOffSfa + kStages * kSfaBytes;
constexpr int kOffBar = kOffSfb + kStages * kSfbBytes;
// full[S], empty[S], acc_full, acc_empty, drain
constexpr int kNumBars = 2 * kStages + 3;
constexpr int kOffTmemSlot = kOffBar + kNumBars * 8;
constexpr int kOffAbort = kOffTmemSlot + 4;
constexpr int kSmemUsed = kOffAbort + 4;
constexpr int kGemmSmemBytes = kSmemUsed + 1024;  // slack to align the base to 1024 bytes

// Output addressing shared by the kernels: C is a row-major view with row stride `ldc` elements
// starting at column `col0` of the buffer at `c`. With n_peer > 0 every tile is also stored, at
// the same offset, into peer[0..n_peer) (other GPUs' buffers mapped into this process, reached
// over NVLink with plain 16-byte stores): the gather of a column-parallel GEMM fused into the
// epilogue. n_peer = 0, ldc = N, col0 = 0 is the ordinary contiguous [M, N] output.
constexpr int kMaxPeers = 7;

struct GemmParams {
  const uint8_t* sfa;
  const uint8_t* sfb;
  void* c;
  int64_t ldc, col0;
  int n_peer;
  void* peer[kMaxPeers];
  const float* alpha;
  int* status;
  int m, n, k;
  int m_tiles, n_tiles, k_tiles;
  int sf_kblocks;    // ceil(K/64): 512-byte scale chunks per 128-row block
  int n_rowblocks;   // ceil(N/128)
  int num_tiles;
  int raster_band;
  int raster_along_m;
  int pol_a, pol_b, pol_sfa, pol_sfb;
  int store_evict_first;
  int pace_ns;
  int tma_b_first;
  // Bytes of one A box of the one-CTA kernel: 128 B x min(128, M rounded up to 8) rows. With
  // fewer than 128 rows of A the box covers only the rows that exist: rows of shared memory
  // beyond it hold stale data, which feeds only output rows >= M, and those are not stored.
  // (A 128-row box over an operand of under 32 rows runs at about half speed on B200.)
  int a_box_bytes;
};

// Linear persistent work index -> (m-tile, n-tile). Bands of `raster_band` tiles along one
// dimension are swept across the other, keeping a band's operand rows hot in L2.
__device__ __forceinline__ void tile_coord(const GemmParams& p, int t, int& mt, int& nt) {
  const int g = p.raster_band > 1 ? p.raster_band : 1;
  if (!p.raster_along_m) {
    const int per_band = g * p.n_tiles;
    const int band = t / per_band;
    const int within = t - band * per_band;
    const int rows = min(g, p.m_tiles - band * g);
    mt = band * g + within % rows;
    nt = within / rows;
  } else {
    const int per_band = g * p.m_tiles;
    const int band = t / per_band;
    const int within = t - band * per_band;
    const int cols = min(g, p.n_tiles - band * g);
    nt = band * g + within % cols;
    mt = within / cols;
  }
}

// Fused gather: copy the 32 output rows a warp has just stored (row0 .. row0 + 31, columns
// [0, cols) of the tile at byte offset `off0` of row row0) from this GPU's buffer into every peer
// buffer. A lane carries 16 bytes, so each warp store writes 512 contiguous bytes of one row over
// NVLink; per-thread stores of a thread's own row would scatter 16-byte pieces over 32 rows. The
// rows are read back through L2 (ld.global.cg), two at a time (more would spill registers of the
// pair kernel).
__device__ __forceinline__ void copy_rows_to_peers(const GemmParams& p, int row0, int cols, size_t off0, int lane) {
  const size_t pitch = static_cast<size_t>(p.ldc) * 2;
  const bool on = lane * 8 < cols;  // 8 columns (16 bytes) per lane
  const int rows = min(32, p.m - row0);
  for (int i0 = 0; i0 < rows; i0 += 2) {
    uint4 v[2];
#pragma unroll
    for (int i = 0; i < 2; ++i)
      if (on && i0 + i < rows)
        v[i] = __ldcg(reinterpret_cast<const uint4*>(static_cast<const uint8_t*>(p.c) + off0 + (i0 + i) * pitch) + lane);
    for (int d = 0; d < p.n_peer; ++d) {
#pragma unroll
      for (int i = 0; i < 2; ++i)
        if (on && i0 + i < rows)
          reinterpret_cast<uint4*>(static_cast<uint8_t*>(p.peer[d]) + off0 + (i0 + i) * pitch)[lane] = v[i];
    }
  }
}

__device__ __forceinline__ uint32_t pack_out(float lo, float hi, bool bf16) {
  if (bf16) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  }
  __half2 v = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

template <bool kBF16>
__global__ void __launch_bounds__(kGemmThreads, 1)
    nvfp4_gemm_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                      const GemmParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint64_t* full = bars;
  uint64_t* empty = bars + kStages;
  uint64_t* acc_full = bars + 2 * kStages;
  uint64_t* acc_empty = acc_full + 1;
  uint64_t* drain = acc_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kOffTmemSlot);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + kOffAbort);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(acc_empty, 4 * 32);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbarrier_init();
    prefetch_tmap(&tmap_a);
    prefetch_tmap(&tmap_b);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // Programmatic dependent launch: set-up overlaps the preceding kernel; global memory is
  // touched only after it has completed (as in the CTA-pair kernel).
  griddep_launch_dependents();
  griddep_wait();

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    // One thread walks the schedule. Warp-wide collectives inside this loop (a divergent wait
    // followed by a shuffle or __syncwarp per k-tile) roughly halve the MMA issue rate.
    if (lane == 0) {
      const uint64_t pol_a = make_policy(p.pol_a);
      const uint64_t pol_b = make_policy(p.pol_b);
      const uint64_t pol_sfa = make_policy(p.pol_sfa);
      const uint64_t pol_sfb = make_policy(p.pol_sfb);
      uint32_t stage = 0, phase = 0;
      uint32_t issued_mask = 0, issued_parity = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < p.num_tiles; t += gridDim.x) {
        int mt, nt;
        tile_coord(p, t, mt, nt);
        const int nrb = min(2, p.n_rowblocks - 2 * nt);
        for (int kt = 0; kt < p.k_tiles; ++kt) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, p.status, kStatusTimeoutEmpty, abort_flag)) {
            ok = false;
            break;
          }
          const int nkb = min(kKBlocksPerTile, p.sf_kblocks - kKBlocksPerTile * kt);
          const uint32_t sf_bytes = static_cast<uint32_t>(nkb * kSfChunk);
          mbar_arrive_expect_tx(&full[stage], p.a_box_bytes + kBBytes + sf_bytes * (1 + nrb));
          uint8_t* sa = smem + kOffA + stage * kABytes;
          uint8_t* sb = smem + kOffB + stage * kBBytes;
          if (p.tma_b_first) {
            tma_load_2d(sb, &tmap_b, kt * kTileKBytes, nt * kTileN, &full[stage], pol_b);
            tma_load_2d(sa, &tmap_a, kt * kTileKBytes, mt * kTileM, &full[stage], pol_a);
          } else {
            tma_load_2d(sa, &tmap_a, kt * kTileKBytes, mt * kTileM, &full[stage], pol_a);
            tma_load_2d(sb, &tmap_b, kt * kTileKBytes, nt * kTileN, &full[stage], pol_b);
          }
          const size_t kb0 = static_cast<size_t>(kKBlocksPerTile) * kt;
          bulk_load(smem + kOffSfa + stage * kSfaBytes,
                    p.sfa + (static_cast<size_t>(mt) * p.sf_kblocks + kb0) * kSfChunk, sf_bytes, &full[stage],
                    pol_sfa);
          for (int rb = 0; rb < nrb; ++rb) {
            bulk_load(smem + kOffSfb + stage * kSfbBytes + rb * (kKBlocksPerTile * kSfChunk),
                      p.sfb + (static_cast<size_t>(2 * nt + rb) * p.sf_kblocks + kb0) * kSfChunk, sf_bytes,
                      &full[stage], pol_sfb);
          }
          issued_mask |= 1u << stage;
          issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (ok) {
        // Tail: wait until the MMA warp has released every stage, so no tcgen05.commit arrival
        // is still in flight when the CTA exits.
        for (int s = 0; s < kStages; ++s) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, p.status, kStatusTimeoutEmpty, abort_flag)) break;
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      } else {
        // Unwind: let the copies already issued land before shared memory goes away.
        for (int s = 0; s < kStages; ++s)
          if (issued_mask & (1u << s))
            mbar_wait(&full[s], (issued_parity >> s) & 1u, p.status, kStatusTimeoutDrain, nullptr);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer (one thread)
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_nvf4(kTileM, kTileN);
      uint32_t stage = 0, phase = 0, acc_phase = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < p.num_tiles; t += gridDim.x) {
        int mt, nt;
        tile_coord(p, t, mt, nt);
        const int nrb = min(2, p.n_rowblocks - 2 * nt);
        if (!mbar_wait(acc_empty, acc_phase ^ 1u, p.status, kStatusTimeoutAccEmpty, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        for (int kt = 0; kt < p.k_tiles; ++kt) {
          if (!mbar_wait(&full[stage], phase, p.status, kStatusTimeoutFull, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const int nkb = min(kKBlocksPerTile, p.sf_kblocks - kKBlocksPerTile * kt);
          const uint32_t sa = smem_u32(smem + kOffA + stage * kABytes);
          const uint32_t sb = smem_u32(smem + kOffB + stage * kBBytes);
          const uint32_t ssfa = smem_u32(smem + kOffSfa + stage * kSfaBytes);
          const uint32_t ssfb = smem_u32(smem + kOffSfb + stage * kSfbBytes);
          const uint32_t tsfa = tmem + kSfaCol + stage * kSfColsPerStage;
          const uint32_t tsfb = tmem + kSfbCol + stage * kSfColsPerStage;
          if (nkb == kKBlocksPerTile && nrb == 2) {
            // Full k-tile: straight-line issue, scale copies interleaved with the MMA that reads
            // them. Runtime-bounded loops between tcgen05 instructions cost ~70% more issue time.
            const uint64_t da = sdesc_kmajor_sw128(sa), db = sdesc_kmajor_sw128(sb);
            const uint64_t dsa = sdesc_sf_chunk(ssfa), dsb = sdesc_sf_chunk(ssfb);
#pragma unroll
            for (int j = 0; j < kKBlocksPerTile; ++j) {
              // descriptor start addresses are in 16-byte units: +32 B per K=64 step, +512 B per chunk
              tc_cp_32x128b_warpx4(tsfa + 4 * j, dsa + 32 * j);
              tc_cp_32x128b_warpx4(tsfb + 8 * j, dsb + 32 * j);
              tc_cp_32x128b_warpx4(tsfb + 8 * j + 4, dsb + 32 * (j + kKBlocksPerTile));
              tc_mma_nvf4(tmem + kAccCol, da + 2 * j, db + 2 * j, idesc, tsfa + 4 * j, tsfb + 8 * j,
                          (kt | j) != 0 ? 1u : 0u);
            }
          } else {
            for (int j = 0; j < nkb; ++j) tc_cp_32x128b_warpx4(tsfa + 4 * j, sdesc_sf_chunk(ssfa + j * kSfChunk));
            for (int rb = 0; rb < nrb; ++rb)
              for (int j = 0; j < nkb; ++j)
                tc_cp_32x128b_warpx4(tsfb + 8 * j + 4 * rb,
                                     sdesc_sf_chunk(ssfb + rb * (kKBlocksPerTile * kSfChunk) + j * kSfChunk));
            for (int j = 0; j < nkb; ++j) {
              tc_mma_nvf4(tmem + kAccCol, sdesc_kmajor_sw128(sa + 32 * j), sdesc_kmajor_sw128(sb + 32 * j), idesc,
                          tsfa + 4 * j, tsfb + 8 * j, (kt | j) != 0 ? 1u : 0u);
            }
          }
          tc_commit(&empty[stage]);
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        tc_commit(acc_full);
        acc_phase ^= 1u;
      }
      if (!ok) {
        // Unwind: wait for the MMAs already issued before TMEM is released.
        tc_commit(drain);
        mbar_wait(drain, 0, p.status, kStatusTimeoutDrain, nullptr);
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------------ epilogue (warps 2-5)
    const int quad = warp & 3;  // TMEM lane quadrant this warp may access
    const int row = quad * 32 + lane;
    const uint32_t tmem_row = tmem + (static_cast<uint32_t>(quad * 32) << 16);
    const float alpha = *p.alpha;
    const bool evict_first = p.store_evict_first != 0;
    uint32_t acc_phase = 0;
    for (int t = blockIdx.x; t < p.num_tiles; t += gridDim.x) {
      int mt, nt;
      tile_coord(p, t, mt, nt);
      if (!mbar_wait(acc_full, acc_phase, p.status, kStatusTimeoutAccFull, abort_flag)) break;
      acc_phase ^= 1u;
      tc_fence_after();
      uint32_t out[kTileN / 2];
#pragma unroll
      for (int ch = 0; ch < kTileN / 32; ++ch) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(tmem_row + kAccCol + ch * 32, r);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 16; ++i)
          out[ch * 16 + i] = pack_out(__fmul_rn(__uint_as_float(r[2 * i]), alpha),
                                      __fmul_rn(__uint_as_float(r[2 * i + 1]), alpha), kBF16);
      }
      tc_fence_before();
      mbar_arrive(acc_empty);

      const int gm = mt * kTileM + row;
      if (gm < p.m) {
        const size_t off = (static_cast<size_t>(gm) * p.ldc + p.col0 + static_cast<size_t>(nt) * kTileN) * 2;
        uint8_t* rowp = reinterpret_cast<uint8_t*>(p.c) + off;
        const int cols_left = p.n - nt * kTileN;
#pragma unroll
        for (int ch = 0; ch < kTileN / 32; ++ch) {
          if (ch * 32 < cols_left) {
            uint32_t v0[8], v1[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              v0[i] = out[ch * 16 + i];
              v1[i] = out[ch * 16 + 8 + i];
            }
            if (evict_first) {
              st_global_v8_ef(rowp + ch * 64, v0);
              st_global_v8_ef(rowp + ch * 64 + 32, v1);
            } else {
              st_global_v8(rowp + ch * 64, v0);
              st_global_v8(rowp + ch * 64 + 32, v1);
            }
            if (p.pace_ns > 0 && ch + 1 < kTileN / 32) __nanosleep(p.pace_ns);
          }
        }
      }
      if (p.n_peer > 0) {
        __threadfence_block();  // this warp's row stores, before its lanes read each other's rows
        __syncwarp();
        const int row0 = mt * kTileM + quad * 32;
        if (row0 < p.m)
          copy_rows_to_peers(p, row0, min(kTileN, p.n - nt * kTileN),
                             (static_cast<size_t>(row0) * p.ldc + p.col0 + static_cast<size_t>(nt) * kTileN) * 2, lane);
      }
    }
  }

  // Peer stores are visible to the other GPUs before this grid is seen as complete.
  if (p.n_peer > 0) __threadfence_system();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

}  // namespace g3
