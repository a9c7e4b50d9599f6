// Persistent NVFP4 block-scaled GEMM on CTA pairs (tcgen05 cta_group::2) for sm_100a.
//
// A cluster of two CTAs on neighbouring SMs computes 256x256 output tiles. CTA r of the pair
// owns output rows [m0 + 128 r, +128) and supplies B rows [n0 + 128 r, +128); one tcgen05.mma
// (M=256, N=256, K=64) issued by CTA 0 reads A and B from both CTAs' shared memory and writes each
// CTA's half of the accumulator into its own TMEM. Compared with one-CTA 128x256 tiles this halves
// the B bytes every SM loads from L2 and reads from shared memory per FLOP.
//
// A stage covers K = 512 (eight 64-element blocks, eight MMAs, 1,032 tensor-pipe cycles: one
// CTA-pair MMA takes 129). Two shared-memory rings feed the MMA: a 3-stage ring of A/B stages
// (64 KiB per CTA) and a 2-slot ring of scale stages (12 KiB). Scales sit in TMEM in two
// 96-column regions used alternately, independent of the A/B stage; the copies into a region wait
// for the MMAs two stages back, the last readers of it. The scale copies bound the main loop: a
// stage needs 24 tcgen05.cp (.32x128b.warpx4, 2 KiB of TMEM writes each), and while MMAs run each
// takes about 52 cycles, about 1,240 cycles per stage.
//
// Roles (per CTA, 10 warps):
//   warp 0      A/B producer, both CTAs: TMA loads of its A and B halves (128 rows x 128 B,
//               128-byte swizzle), completing on CTA 0's "full" barrier of the stage;
//   warp 2      scale producer, both CTAs: TMA loads of its 128 rows of A scales and all 256 rows
//               of B scales (3-D tensor maps over the swizzled layout), on CTA 0's "sf_full";
//   warp 1      TMEM owner in both CTAs; in CTA 0 the MMA issuer: one tcgen05.mma (cta_group::2)
//               per 64-element block after one wait per stage; one multicast commit releases the
//               A/B stage in both CTAs and, per tile, hands the accumulator to both epilogues;
//   warps 3,4,9 in CTA 0, scale copies into both TMEMs (tcgen05.cp cta_group::2): warp 3 one
//               A-scale chunk per 64-element block, warps 4 and 9 the B-scale chunks of tile
//               rows 0-127 and 128-255. A copy takes its issuing thread about 51 cycles, so the
//               three copies of a block are spread over three threads and the MMA thread issues
//               only MMAs (with one thread for both B chunks, that thread set the pace). A copy
//               warp hands its TMEM region to the MMA thread once the copies are issued (fence +
//               mbarrier arrive; warp 3 first waits for the stage's A/B data) and frees the
//               shared-memory slot through a commit when they have completed;
//   warps 5-8   epilogue, both CTAs: TMEM -> registers -> x alpha -> FP16/BF16, accumulator
//               released to CTA 0's MMA warp, then 256-bit row stores.
// No TMA multicast is used: every CTA loads what it needs itself. The accumulation order per
// output element is k = 0, 64, 128, ... as in the one-CTA kernel, so both produce the same bits.
#pragma once
#include "gemm_kernel.cuh"

namespace g3 {

constexpr int kPairTileM = 256;
constexpr int kPairTileN = 256;
constexpr int kPairKBlocks = 8;                                // 64-element blocks per stage: K = 512
constexpr int kPairKAtoms = kPairKBlocks / kKBlocksPerTile;    // 128-byte swizzle atoms per row (2)
constexpr int kPairStages = 3;     // A/B ring
constexpr int kPairSfSlots = 2;    // scale ring
constexpr int kPairSfRegions = 2;  // TMEM scale regions
constexpr int kPairAtomBytes = 128 * kTileKBytes;              // 128 rows x 128 bytes
constexpr int kPairABytes = kPairKAtoms * kPairAtomBytes;      // this CTA's 128 A rows
constexpr int kPairBBytes = kPairKAtoms * kPairAtomBytes;      // this CTA's 128 B rows
constexpr int kPairSfaBytes = kPairKBlocks * kSfChunk;         // 128 rows x 32 scales
constexpr int kPairSfbBytes = 2 * kPairKBlocks * kSfChunk;     // 256 rows x 32 scales
constexpr uint32_t kPairAbTx = 2u * (kPairABytes + kPairBBytes);     // both CTAs, on CTA 0's barrier
constexpr uint32_t kPairSfTx = 2u * (kPairSfaBytes + kPairSfbBytes);

constexpr int kPairOffA = 0;
constexpr int kPairOffB = kPairOffA + kPairStages * kPairABytes;
constexpr int kPairOffSfa = kPairOffB + kPairStages * kPairBBytes;
constexpr int kPairOffSfb = kPairOffSfa + kPairSfSlots * kPairSfaBytes;
constexpr int kPairOffBar = kPairOffSfb + kPairSfSlots * kPairSfbBytes;
// full[S], empty[S], ready[S], sf_full[Q], sf_empty[Q], acc_full, acc_empty, drain[4] (one per
// tcgen05 issuer)
constexpr int kPairNumBars = 3 * kPairStages + 2 * kPairSfSlots + 6;
constexpr int kPairCopyWarps = 3;  // A scales, B scales rows 0-127, B scales rows 128-255
constexpr int kPairThreads = 320;
constexpr int kPairOffTmemSlot = kPairOffBar + kPairNumBars * 8;
constexpr int kPairOffAbort = kPairOffTmemSlot + 4;
constexpr int kPairSmemBytes = kPairOffAbort + 4 + 1024;

// TMEM columns: accumulator [0, 256); two scale regions of 32 A-scale + 64 B-scale columns.
constexpr int kPairSfaCol = 256;
constexpr int kPairSfColsPerStage = 4 * kPairKBlocks + 8 * kPairKBlocks;
static_assert(kPairSfaCol + kPairSfRegions * kPairSfColsPerStage <= kTmemCols, "pair scales do not fit in TMEM");
static_assert(kPairSmemBytes <= 232448, "pair kernel exceeds shared memory");

// Epilogue drain of 32-column chunks [kC0, kC0 + kN) of one warp's accumulator rows in one TMEM
// round trip: kN loads in flight, one wait, then x alpha (paired FP32 multiplies, the same IEEE
// products as single ones) and packing to FP16/BF16 pairs.
template <int kC0, int kN, bool kBF16>
__device__ __forceinline__ void pair_drain_chunks(uint32_t taddr, float alpha, uint32_t (&out)[kPairTileN / 2]) {
  uint32_t r[kN][32];
#pragma unroll
  for (int c = 0; c < kN; ++c) tmem_ld_32x32b_x32(taddr + (kC0 + c) * 32, r[c]);
  tmem_ld_wait();
  const float2 alpha2 = make_float2(alpha, alpha);
#pragma unroll
  for (int c = 0; c < kN; ++c)
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const float2 v = __fmul2_rn(make_float2(__uint_as_float(r[c][2 * i]), __uint_as_float(r[c][2 * i + 1])), alpha2);
      out[(kC0 + c) * 16 + i] = pack_out(v.x, v.y, kBF16);
    }
}

template <bool kBF16>
__global__ void __launch_bounds__(kPairThreads, 1)
    nvfp4_gemm_pair_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                           const __grid_constant__ CUtensorMap tmap_sfa, const __grid_constant__ CUtensorMap tmap_sfb,
                           const GemmParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kPairOffBar);
  uint64_t* full = bars;
  uint64_t* empty = full + kPairStages;
  uint64_t* ready = empty + kPairStages;  // stage's scales copied and its A/B data landed
  uint64_t* sf_full = ready + kPairStages;
  uint64_t* sf_empty = sf_full + kPairSfSlots;
  uint64_t* acc_full = sf_empty + kPairSfSlots;
  uint64_t* acc_empty = acc_full + 1;
  uint64_t* drain = acc_full + 2;  // [0] MMA, [1] A scales, [2] B scales 0-127, [3] B scales 128-255
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kPairOffTmemSlot);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + kPairOffAbort);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int k_iters = (p.sf_kblocks + kPairKBlocks - 1) / kPairKBlocks;  // stages per tile
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int pair = blockIdx.x >> 1;
  const int num_pairs = gridDim.x >> 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kPairStages; ++s) {
      mbar_init(&full[s], 1);   // one arrive.expect_tx by CTA 0's A/B producer + both CTAs' bytes
      mbar_init(&empty[s], 1);  // one commit from CTA 0's MMA thread
      mbar_init(&ready[s], kPairCopyWarps);  // one arrive from each copy warp
    }
    for (int q = 0; q < kPairSfSlots; ++q) {
      mbar_init(&sf_full[q], 1);   // one arrive.expect_tx by CTA 0's scale producer
      mbar_init(&sf_empty[q], kPairCopyWarps);  // one commit from each copy warp (multicast to both CTAs)
    }
    mbar_init(acc_full, 1);
    mbar_init(acc_empty, 2 * 4);  // every epilogue warp of both CTAs
    for (int d = 0; d < 1 + kPairCopyWarps; ++d) mbar_init(&drain[d], 1);
    *abort_flag = 0;
    fence_mbarrier_init();
    prefetch_tmap(&tmap_a);
    prefetch_tmap(&tmap_b);
    prefetch_tmap(&tmap_sfa);
    prefetch_tmap(&tmap_sfb);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();  // barriers of both CTAs initialised, TMEM allocated in both
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // Programmatic dependent launch (nvfp4_gemm_cute/kernel.py:524, :910-911): the set-up above
  // overlaps the tail of the preceding kernel on the stream; every thread waits here, before
  // its first global read or write, until that kernel has completed and its memory is visible
  // (at once for a plain launch). The next kernel may be scheduled at once: with this CTA's
  // shared memory it can only become resident on SMs that this grid has left.
  griddep_launch_dependents();
  griddep_wait();

  // CTA 0's barriers as seen from either CTA of the pair.
  const uint32_t full0 = mapa_shared(smem_u32(full), 0);
  const uint32_t sf_full0 = mapa_shared(smem_u32(sf_full), 0);
  const uint32_t acc_empty0 = mapa_shared(smem_u32(acc_empty), 0);

  if (warp == 0) {
    // ------------------------------------------------------------------ A/B producer (both CTAs)
    // One thread walks the schedule (warp collectives inside the loop halve the issue rate).
    if (lane == 0) {
      const uint64_t pol_a = make_policy(p.pol_a);
      const uint64_t pol_b = make_policy(p.pol_b);
      uint32_t stage = 0, phase = 0;
      uint32_t issued_mask = 0, issued_parity = 0;
      bool ok = true;
      for (int t = pair; ok && t < p.num_tiles; t += num_pairs) {
        int mt, nt;
        tile_coord(p, t, mt, nt);
        const int row_a = mt * kPairTileM + 128 * static_cast<int>(rank);
        const int row_b = nt * kPairTileN + 128 * static_cast<int>(rank);
        for (int kt = 0; kt < k_iters; ++kt) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, p.status, kStatusTimeoutEmpty, abort_flag)) {
            ok = false;
            break;
          }
          const uint32_t bar = full0 + 8u * stage;
          if (leader) mbar_arrive_expect_tx(&full[stage], kPairAbTx);
          uint8_t* sa = smem + kPairOffA + stage * kPairABytes;
          uint8_t* sb = smem + kPairOffB + stage * kPairBBytes;
          // one 128-byte swizzle atom (256 elements of K) per box; the stage holds kPairKAtoms
          const int x0 = kt * kPairKAtoms * kTileKBytes;
          if (p.tma_b_first) {
#pragma unroll
            for (int h = 0; h < kPairKAtoms; ++h)
              tma_load_2d_pair(sb + h * kPairAtomBytes, &tmap_b, x0 + h * kTileKBytes, row_b, bar, pol_b);
#pragma unroll
            for (int h = 0; h < kPairKAtoms; ++h)
              tma_load_2d_pair(sa + h * kPairAtomBytes, &tmap_a, x0 + h * kTileKBytes, row_a, bar, pol_a);
          } else {
#pragma unroll
            for (int h = 0; h < kPairKAtoms; ++h) {
              tma_load_2d_pair(sa + h * kPairAtomBytes, &tmap_a, x0 + h * kTileKBytes, row_a, bar, pol_a);
              tma_load_2d_pair(sb + h * kPairAtomBytes, &tmap_b, x0 + h * kTileKBytes, row_b, bar, pol_b);
            }
          }
          issued_mask |= 1u << stage;
          issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
          if (++stage == kPairStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (ok) {
        // Tail: every stage released by CTA 0's MMA thread, so no commit is still in flight.
        for (int s = 0; s < kPairStages; ++s) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, p.status, kStatusTimeoutEmpty, abort_flag)) break;
          if (++stage == kPairStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      } else if (leader) {
        for (int s = 0; s < kPairStages; ++s)
          if (issued_mask & (1u << s))
            mbar_wait(&full[s], (issued_parity >> s) & 1u, p.status, kStatusTimeoutDrain, nullptr);
      }
    }
    __syncwarp();
  } else if (warp == 2) {
    // ------------------------------------------------------------------ scale producer (both CTAs)
    if (lane == 0) {
      const uint64_t pol_sfa = make_policy(p.pol_sfa);
      const uint64_t pol_sfb = make_policy(p.pol_sfb);
      uint32_t slot = 0, phase = 0;
      uint32_t issued_mask = 0, issued_parity = 0;
      bool ok = true;
      for (int t = pair; ok && t < p.num_tiles; t += num_pairs) {
        int mt, nt;
        tile_coord(p, t, mt, nt);
        const int rb_a = (mt * kPairTileM + 128 * static_cast<int>(rank)) >> 7;
        for (int kt = 0; kt < k_iters; ++kt) {
          if (!mbar_wait(&sf_empty[slot], phase ^ 1u, p.status, kStatusTimeoutEmpty, abort_flag)) {
            ok = false;
            break;
          }
          const uint32_t bar = sf_full0 + 8u * slot;
          if (leader) mbar_arrive_expect_tx(&sf_full[slot], kPairSfTx);
          // scale chunks: {512-byte chunk, 64-element block, 128-row block}
          const int kb0 = kPairKBlocks * kt;
          tma_load_3d_pair(smem + kPairOffSfa + slot * kPairSfaBytes, &tmap_sfa, 0, kb0, rb_a, bar, pol_sfa);
          tma_load_3d_pair(smem + kPairOffSfb + slot * kPairSfbBytes, &tmap_sfb, 0, kb0, 2 * nt, bar, pol_sfb);
          issued_mask |= 1u << slot;
          issued_parity = (issued_parity & ~(1u << slot)) | (phase << slot);
          if (++slot == kPairSfSlots) {
            slot = 0;
            phase ^= 1u;
          }
        }
      }
      if (ok) {
        for (int q = 0; q < kPairSfSlots; ++q) {
          if (!mbar_wait(&sf_empty[slot], phase ^ 1u, p.status, kStatusTimeoutEmpty, abort_flag)) break;
          if (++slot == kPairSfSlots) {
            slot = 0;
            phase ^= 1u;
          }
        }
      } else if (leader) {
        for (int q = 0; q < kPairSfSlots; ++q)
          if (issued_mask & (1u << q))
            mbar_wait(&sf_full[q], (issued_parity >> q) & 1u, p.status, kStatusTimeoutDrain, nullptr);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer (CTA 0, one thread)
    if (leader && lane == 0) {
      constexpr uint32_t idesc = idesc_nvf4(kPairTileM, kPairTileN);
      const uint32_t empty_off = smem_u32(empty), accf_off = smem_u32(acc_full);
      uint32_t stage = 0, phase = 0, acc_phase = 0, region = 0;
      bool ok = true;
      for (int t = pair; ok && t < p.num_tiles; t += num_pairs) {
        if (!mbar_wait(acc_empty, acc_phase ^ 1u, p.status, kStatusTimeoutAccEmpty, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        for (int kt = 0; kt < k_iters; ++kt) {
          if (!mbar_wait(&ready[stage], phase, p.status, kStatusTimeoutFull, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const int nkb = min(kPairKBlocks, p.sf_kblocks - kPairKBlocks * kt);
          const uint64_t da = sdesc_kmajor_sw128(smem_u32(smem + kPairOffA + stage * kPairABytes));
          const uint64_t db = sdesc_kmajor_sw128(smem_u32(smem + kPairOffB + stage * kPairBBytes));
          const uint32_t tsfa = tmem + kPairSfaCol + region * kPairSfColsPerStage;
          const uint32_t tsfb = tsfa + 4 * kPairKBlocks;
          // block j: swizzle atom j / 4 (kPairAtomBytes apart), 32-byte K step j % 4 inside it
          if (nkb == kPairKBlocks) {
#pragma unroll
            for (int j = 0; j < kPairKBlocks; ++j) {
              const uint32_t off = (j >> 2) * (kPairAtomBytes >> 4) + 2 * (j & 3);
              tc_mma_nvf4_pair(tmem + kAccCol, da + off, db + off, idesc, tsfa + 4 * j, tsfb + 8 * j,
                               (kt | j) != 0 ? 1u : 0u);
            }
          } else {
            for (int j = 0; j < nkb; ++j) {
              const uint32_t off = (j >> 2) * (kPairAtomBytes >> 4) + 2 * (j & 3);
              tc_mma_nvf4_pair(tmem + kAccCol, da + off, db + off, idesc, tsfa + 4 * j, tsfb + 8 * j,
                               (kt | j) != 0 ? 1u : 0u);
            }
          }
          tc_commit_pair_mc(empty_off + 8u * stage, 0x3);
          if (++stage == kPairStages) {
            stage = 0;
            phase ^= 1u;
          }
          if (++region == kPairSfRegions) region = 0;
        }
        if (!ok) break;
        tc_commit_pair_mc(accf_off, 0x3);
        acc_phase ^= 1u;
      }
      if (!ok) {
        tc_commit_pair(smem_u32(&drain[0]));
        mbar_wait(&drain[0], 0, p.status, kStatusTimeoutDrain, nullptr);
      }
    }
    __syncwarp();
  } else if (warp == 3 || warp == 4 || warp == 9) {
    // ------------------------------------------------------------------ scale copies (CTA 0)
    // Warp 3 copies the A scales (one 512-byte chunk per 64-element block), warps 4 and 9 the B
    // scales of tile rows 0-127 and 128-255. Stage iteration g lands in scale slot g % Q and is
    // copied into TMEM region g % R once the MMAs of iteration g - R, the last readers of that
    // region, have completed: completion number (g - R) / S of the empty barrier of A/B stage
    // (g - R) % S. That barrier cannot run two completions ahead, since iteration g + 1 needs
    // these copies first.
    if (leader && lane == 0) {
      const bool is_a = warp == 3;
      const int half = warp == 9 ? 1 : 0;  // B-scale copy warps: which 128 rows of the tile
      const int role = is_a ? 1 : 2 + half;  // drain barrier index
      const uint32_t sfe_off = smem_u32(sf_empty);
      uint32_t stage = 0, phase = 0, slot = 0, sphase = 0, region = 0;
      uint32_t lag_stage = 0, lag_phase = 0;  // A/B stage and completion parity of iteration g - R
      int it = 0;
      bool ok = true;
      for (int t = pair; ok && t < p.num_tiles; t += num_pairs) {
        for (int kt = 0; kt < k_iters; ++kt, ++it) {
          if (!mbar_wait(&sf_full[slot], sphase, p.status, kStatusTimeoutFull, abort_flag)) {
            ok = false;
            break;
          }
          if (it >= kPairSfRegions) {
            if (!mbar_wait(&empty[lag_stage], lag_phase, p.status, kStatusTimeoutEmpty, abort_flag)) {
              ok = false;
              break;
            }
            if (++lag_stage == kPairStages) {
              lag_stage = 0;
              lag_phase ^= 1u;
            }
          }
          tc_fence_after();
          const int nkb = min(kPairKBlocks, p.sf_kblocks - kPairKBlocks * kt);
          const uint32_t tsfa = tmem + kPairSfaCol + region * kPairSfColsPerStage;
          const uint32_t tsfb = tsfa + 4 * kPairKBlocks;
          if (is_a) {
            const uint64_t dsa = sdesc_sf_chunk(smem_u32(smem + kPairOffSfa + slot * kPairSfaBytes));
            if (nkb == kPairKBlocks) {
#pragma unroll
              for (int j = 0; j < kPairKBlocks; ++j) tc_cp_32x128b_warpx4_pair(tsfa + 4 * j, dsa + 32 * j);
            } else {
              for (int j = 0; j < nkb; ++j) tc_cp_32x128b_warpx4_pair(tsfa + 4 * j, dsa + 32 * j);
            }
          } else {
            const uint64_t dsb =
                sdesc_sf_chunk(smem_u32(smem + kPairOffSfb + slot * kPairSfbBytes)) + 32 * kPairKBlocks * half;
            const uint32_t tb = tsfb + 4 * half;
            if (nkb == kPairKBlocks) {
#pragma unroll
              for (int j = 0; j < kPairKBlocks; ++j) tc_cp_32x128b_warpx4_pair(tb + 8 * j, dsb + 32 * j);
            } else {
              for (int j = 0; j < nkb; ++j) tc_cp_32x128b_warpx4_pair(tb + 8 * j, dsb + 32 * j);
            }
          }
          // The TMEM region goes to the MMA thread as soon as the copies are issued: the fence
          // orders them before this arrive, the MMA thread's after_thread_sync fence orders its
          // MMAs after it, and the tensor pipe runs them in that order. Warp 3 also waits for the
          // stage's A/B data, so the MMA thread waits on one barrier per stage. The
          // shared-memory slot is freed only when the copies have completed.
          tc_fence_before();
          if (is_a && !mbar_wait(&full[stage], phase, p.status, kStatusTimeoutFull, abort_flag)) {
            ok = false;
            break;
          }
          mbar_arrive(&ready[stage]);
          tc_commit_pair_mc(sfe_off + 8u * slot, 0x3);
          if (++stage == kPairStages) {
            stage = 0;
            phase ^= 1u;
          }
          if (++slot == kPairSfSlots) {
            slot = 0;
            sphase ^= 1u;
          }
          if (++region == kPairSfRegions) region = 0;
        }
      }
      if (!ok) {
        tc_commit_pair(smem_u32(&drain[role]));
        mbar_wait(&drain[role], 0, p.status, kStatusTimeoutDrain, nullptr);
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------------ epilogue (both CTAs)
    const int quad = warp & 3;
    const int row = quad * 32 + lane;
    const uint32_t tmem_row = tmem + (static_cast<uint32_t>(quad * 32) << 16);
    const float alpha = *p.alpha;
    const bool evict_first = p.store_evict_first != 0;
    uint32_t acc_phase = 0;
    for (int t = pair; t < p.num_tiles; t += num_pairs) {
      int mt, nt;
      tile_coord(p, t, mt, nt);
      if (!mbar_wait(acc_full, acc_phase, p.status, kStatusTimeoutAccFull, abort_flag)) break;
      acc_phase ^= 1u;
      tc_fence_after();
      uint32_t out[kPairTileN / 2];
      // The MMA thread idles until the accumulator is drained, so the drain takes three TMEM
      // round trips (96, 96 and 64 columns), as many loads in flight per wait as the registers
      // allow beside the packed output.
      pair_drain_chunks<0, 3, kBF16>(tmem_row + kAccCol, alpha, out);
      pair_drain_chunks<3, 3, kBF16>(tmem_row + kAccCol, alpha, out);
      pair_drain_chunks<6, 2, kBF16>(tmem_row + kAccCol, alpha, out);
      // One arrive per warp once all its lanes' loads have completed: at CTA scope in CTA 0, and
      // relaxed at cluster scope from CTA 1 (per-thread release arrives cost 6 us at 8192^3).
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (leader)
          mbar_arrive(acc_empty);
        else
          mbar_arrive_relaxed_cluster(acc_empty0);
      }

      const int gm = mt * kPairTileM + 128 * static_cast<int>(rank) + row;
      if (gm < p.m) {
        const size_t off = (static_cast<size_t>(gm) * p.ldc + p.col0 + static_cast<size_t>(nt) * kPairTileN) * 2;
        uint8_t* rowp = reinterpret_cast<uint8_t*>(p.c) + off;
        const int cols_left = p.n - nt * kPairTileN;
#pragma unroll
        for (int ch = 0; ch < kPairTileN / 32; ++ch) {
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
            if (p.pace_ns > 0 && ch + 1 < kPairTileN / 32) __nanosleep(p.pace_ns);
          }
        }
      }
      if (p.n_peer > 0) {
        __threadfence_block();  // this warp's row stores, before its lanes read each other's rows
        __syncwarp();
        const int row0 = mt * kPairTileM + 128 * static_cast<int>(rank) + quad * 32;
        if (row0 < p.m)
          copy_rows_to_peers(p, row0, min(kPairTileN, p.n - nt * kPairTileN),
                             (static_cast<size_t>(row0) * p.ldc + p.col0 + static_cast<size_t>(nt) * kPairTileN) * 2,
                             lane);
      }
    }
  }

  // Peer stores are visible to the other GPUs before this grid is seen as complete.
  if (p.n_peer > 0) __threadfence_system();
  tc_fence_before();
  cluster_sync();  // no CTA leaves while its peer may still signal its barriers
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, kTmemCols);
  }
}

}  // namespace g3
