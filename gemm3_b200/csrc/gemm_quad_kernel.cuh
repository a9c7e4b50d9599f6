// Persistent NVFP4 block-scaled GEMM on clusters of two CTA pairs that share their A tiles
// (sm_100a). The CTA-pair kernel (gemm_pair_kernel.cuh) reads every A and B byte of a 256x256 tile
// from L2 once per pair; at 8192^3 that is 2.3 GB of L2 -> SM traffic per GEMM for 76 MB of
// operands, and the feed, not the tensor pipe, sets its pace. Here a cluster of four CTAs runs two
// pairs on neighbouring column tiles of the same 256 rows: pair 0 (CTAs 0, 1) computes tile
// (m, 2j) and pair 1 (CTAs 2, 3) tile (m, 2j + 1). CTA r and CTA r ^ 2 need the same 128 rows of
// A at every stage, so each loads one of the stage's two 128-byte K atoms of them from global
// memory and pushes it into the other's shared memory with a bulk shared::cta -> shared::cluster
// copy (no TMA multicast). A's L2 reads halve, B's stay: about 21 % less L2 -> SM traffic per
// FLOP, scale factors included.
//
// Per CTA and A/B stage s (K = 512: two swizzle atoms of 128 rows x 128 bytes per operand):
//   own[s]    the CTA's own A atom landed (TMA, 16 KiB);
//   full[s]   its two B atoms (TMA, 32 KiB) and the A atom pushed by CTA r ^ 2 (16 KiB) landed;
//   empty[s]  both pairs' MMAs of stage s have completed (two commits, one per pair leader,
//             each multicast to all four CTAs). Only then is stage s free in every CTA at once:
//             its own atom has also been read by the push (the other pair consumed it), and the
//             other pair's push may land in it again.
//   ready[s]  (pair leader) the stage's scales are in TMEM and both CTAs of the pair hold their
//             whole stage: the leader's warp 3 waits own/full locally, the other CTA's warp 3
//             waits them in its CTA and arrives on the leader's ready[s] across the cluster.
// The scale path (warp 2, the three copy warps, two TMEM scale regions), the MMA issue and the
// epilogue are the CTA-pair kernel's, per pair. The accumulation order per output element is the
// same MMA chain, so the output bits equal the pair kernel's.
//
// Roles (per CTA, 11 warps): 0 A/B producer; 1 TMEM owner and, in pair leaders, the MMA issuer;
// 2 scale producer; 3, 4, 9 scale copies (pair leaders), warp 3 also the pair relay in the other
// CTA; 5-8 epilogue; 10 the A-atom push.
#pragma once
#include "gemm_pair_kernel.cuh"

namespace g3 {

constexpr int kQuadThreads = 352;
constexpr int kQuadAtomBytes = kPairAtomBytes;  // one A atom: 128 rows x 128 bytes
// full[S], own[S], empty[S], ready[S], sf_full[Q], sf_empty[Q], acc_full, acc_empty, drain[4]
constexpr int kQuadNumBars = 4 * kPairStages + 2 * kPairSfSlots + 6;
constexpr int kQuadOffBar = kPairOffBar;
constexpr int kQuadOffTmemSlot = kQuadOffBar + kQuadNumBars * 8;
constexpr int kQuadOffAbort = kQuadOffTmemSlot + 4;
constexpr int kQuadSmemBytes = kQuadOffAbort + 4 + 1024;
static_assert(kQuadSmemBytes <= 232448, "quad kernel exceeds shared memory");
constexpr uint32_t kQuadOwnTx = kQuadAtomBytes;                 // own A atom
constexpr uint32_t kQuadFullTx = kPairBBytes + kQuadAtomBytes;  // both B atoms + the pushed A atom

// Waits on a barrier that other CTAs of the cluster arrive on: acquire at cluster scope.
__device__ __forceinline__ bool mbar_try_wait_cluster(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity, int* status, int code,
                                                  volatile int* abort_flag) {
  const uint32_t a = smem_u32(bar);
  if (mbar_try_wait_cluster(a, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  uint32_t spins = 0;
  while (true) {
    if (mbar_try_wait_cluster(a, parity)) return true;
    if ((++spins & 255u) == 0u) {
      if (abort_flag != nullptr && *abort_flag) return false;
      if (globaltimer_ns() - t0 > kWaitTimeoutNs) {
        record_status(status, code);
        if (abort_flag != nullptr) *abort_flag = 1;
        return false;
      }
    }
  }
}

// Bulk copy of `bytes` from this CTA's shared memory to shared memory of another CTA of the
// cluster (dst_cluster, a shared::cluster address), counted on the destination CTA's mbarrier.
__device__ __forceinline__ void bulk_push_cluster(uint32_t dst_cluster, const void* src, uint32_t bytes,
                                                  uint32_t bar_cluster) {
  asm volatile(
      "cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          dst_cluster),
      "r"(smem_u32(src)), "r"(bytes), "r"(bar_cluster)
      : "memory");
}

// Linear super-tile index -> (m-tile, column-pair index), the band raster of tile_coord over
// ceil(n_tiles / 2) column pairs.
__device__ __forceinline__ void quad_tile_coord(const GemmParams& p, int t, int& mt, int& ntp) {
  const int n_pairs = (p.n_tiles + 1) >> 1;
  const int g = p.raster_band > 1 ? p.raster_band : 1;
  if (!p.raster_along_m) {
    const int per_band = g * n_pairs;
    const int band = t / per_band;
    const int within = t - band * per_band;
    const int rows = min(g, p.m_tiles - band * g);
    mt = band * g + within % rows;
    ntp = within / rows;
  } else {
    const int per_band = g * p.m_tiles;
    const int band = t / per_band;
    const int within = t - band * per_band;
    const int cols = min(g, n_pairs - band * g);
    ntp = band * g + within % cols;
    mt = within / cols;
  }
}

template <bool kBF16>
__global__ void __launch_bounds__(kQuadThreads, 1)
    nvfp4_gemm_quad_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                           const __grid_constant__ CUtensorMap tmap_sfa, const __grid_constant__ CUtensorMap tmap_sfb,
                           const GemmParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kQuadOffBar);
  uint64_t* full = bars;
  uint64_t* own = full + kPairStages;
  uint64_t* empty = own + kPairStages;
  uint64_t* ready = empty + kPairStages;
  uint64_t* sf_full = ready + kPairStages;
  uint64_t* sf_empty = sf_full + kPairSfSlots;
  uint64_t* acc_full = sf_empty + kPairSfSlots;
  uint64_t* acc_empty = acc_full + 1;
  uint64_t* drain = acc_full + 2;  // [0] MMA, [1] A scales, [2] B scales 0-127, [3] B scales 128-255
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kQuadOffTmemSlot);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + kQuadOffAbort);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int k_iters = (p.sf_kblocks + kPairKBlocks - 1) / kPairKBlocks;
  const uint32_t crank = cluster_ctarank();  // 0..3
  const uint32_t prank = crank & 1u;         // rank inside the CTA pair
  const uint32_t pid = crank >> 1;           // which pair of the cluster
  const bool leader = prank == 0;
  const uint32_t lead_rank = crank & ~1u;
  const uint16_t pair_mask = static_cast<uint16_t>(0x3u << (2 * pid));
  const int cluster = blockIdx.x >> 2;
  const int num_clusters = gridDim.x >> 2;
  const int my_atom = static_cast<int>(pid);  // the A atom of each stage this CTA loads itself

  if (threadIdx.x == 0) {
    for (int s = 0; s < kPairStages; ++s) {
      mbar_init(&full[s], 1);   // arrive.expect_tx by this CTA's producer + TMA B + pushed A bytes
      mbar_init(&own[s], 1);    // arrive.expect_tx by this CTA's producer + its own A atom
      mbar_init(&empty[s], 2);  // one commit from each pair leader's MMA thread
      mbar_init(&ready[s], kPairCopyWarps + 1);  // the leader's copy warps + the other CTA's relay
    }
    for (int q = 0; q < kPairSfSlots; ++q) {
      mbar_init(&sf_full[q], 1);
      mbar_init(&sf_empty[q], kPairCopyWarps);
    }
    mbar_init(acc_full, 1);
    mbar_init(acc_empty, 2 * 4 * 32);
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
  cluster_sync();  // every CTA's barriers initialised and TMEM allocated before any remote signal
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  griddep_launch_dependents();
  griddep_wait();

  const uint32_t sf_full_lead = mapa_shared(smem_u32(sf_full), lead_rank);
  const uint32_t acc_empty_lead = mapa_shared(smem_u32(acc_empty), lead_rank);
  const uint32_t ready_lead = mapa_shared(smem_u32(ready), lead_rank);

  if (warp == 0) {
    // ------------------------------------------------------------------ A/B producer (every CTA)
    if (lane == 0) {
      const uint64_t pol_a = make_policy(p.pol_a);
      const uint64_t pol_b = make_policy(p.pol_b);
      uint32_t stage = 0, phase = 0;
      uint32_t issued_mask = 0, issued_parity = 0;
      bool ok = true;
      for (int t = cluster; ok && t < p.num_tiles; t += num_clusters) {
        int mt, ntp;
        quad_tile_coord(p, t, mt, ntp);
        const int nt = 2 * ntp + static_cast<int>(pid);
        const int row_a = mt * kPairTileM + 128 * static_cast<int>(prank);
        const int row_b = nt * kPairTileN + 128 * static_cast<int>(prank);
        for (int kt = 0; kt < k_iters; ++kt) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, p.status, kStatusTimeoutEmpty, abort_flag)) {
            ok = false;
            break;
          }
          uint8_t* sa = smem + kPairOffA + stage * kPairABytes;
          uint8_t* sb = smem + kPairOffB + stage * kPairBBytes;
          const int x0 = kt * kPairKAtoms * kTileKBytes;
          mbar_arrive_expect_tx(&own[stage], kQuadOwnTx);
          tma_load_2d(sa + my_atom * kQuadAtomBytes, &tmap_a, x0 + my_atom * kTileKBytes, row_a, &own[stage], pol_a);
          mbar_arrive_expect_tx(&full[stage], kQuadFullTx);
#pragma unroll
          for (int h = 0; h < kPairKAtoms; ++h)
            tma_load_2d(sb + h * kPairAtomBytes, &tmap_b, x0 + h * kTileKBytes, row_b, &full[stage], pol_b);
          issued_mask |= 1u << stage;
          issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
          if (++stage == kPairStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (ok) {
        // Tail: every stage released by both pairs, so no commit or push is still in flight.
        for (int s = 0; s < kPairStages; ++s) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, p.status, kStatusTimeoutEmpty, abort_flag)) break;
          if (++stage == kPairStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      } else {
        // Unwind: let the loads already issued, and the pushes into this CTA, land.
        for (int s = 0; s < kPairStages; ++s)
          if (issued_mask & (1u << s)) {
            mbar_wait(&own[s], (issued_parity >> s) & 1u, p.status, kStatusTimeoutDrain, nullptr);
            mbar_wait(&full[s], (issued_parity >> s) & 1u, p.status, kStatusTimeoutDrain, nullptr);
          }
      }
    }
    __syncwarp();
  } else if (warp == 10) {
    // ------------------------------------------------------------------ A-atom push (every CTA)
    // Once this CTA's own atom of stage s has landed, copy it into the same place in CTA r ^ 2,
    // whose stage s is free too (own[s] follows empty[s], which both pairs released).
    if (lane == 0) {
      const uint32_t peer = crank ^ 2u;
      const uint32_t full_peer = mapa_shared(smem_u32(full), peer);
      const uint32_t a_peer = mapa_shared(smem_u32(smem + kPairOffA), peer);
      uint32_t stage = 0, phase = 0;
      bool ok = true;
      for (int t = cluster; ok && t < p.num_tiles; t += num_clusters) {
        for (int kt = 0; kt < k_iters; ++kt) {
          if (!mbar_wait(&own[stage], phase, p.status, kStatusTimeoutFull, abort_flag)) {
            ok = false;
            break;
          }
          const uint32_t off = stage * kPairABytes + my_atom * kQuadAtomBytes;
          bulk_push_cluster(a_peer + off, smem + kPairOffA + off, kQuadAtomBytes, full_peer + 8u * stage);
          if (++stage == kPairStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    }
    __syncwarp();
  } else if (warp == 2) {
    // ------------------------------------------------------------------ scale producer (every CTA)
    if (lane == 0) {
      const uint64_t pol_sfa = make_policy(p.pol_sfa);
      const uint64_t pol_sfb = make_policy(p.pol_sfb);
      uint32_t slot = 0, phase = 0;
      uint32_t issued_mask = 0, issued_parity = 0;
      bool ok = true;
      for (int t = cluster; ok && t < p.num_tiles; t += num_clusters) {
        int mt, ntp;
        quad_tile_coord(p, t, mt, ntp);
        const int nt = 2 * ntp + static_cast<int>(pid);
        const int rb_a = (mt * kPairTileM + 128 * static_cast<int>(prank)) >> 7;
        for (int kt = 0; kt < k_iters; ++kt) {
          if (!mbar_wait(&sf_empty[slot], phase ^ 1u, p.status, kStatusTimeoutEmpty, abort_flag)) {
            ok = false;
            break;
          }
          const uint32_t bar = sf_full_lead + 8u * slot;
          if (leader) mbar_arrive_expect_tx(&sf_full[slot], kPairSfTx);
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
    // ------------------------------------------------------------------ MMA issuer (pair leaders)
    if (leader && lane == 0) {
      constexpr uint32_t idesc = idesc_nvf4(kPairTileM, kPairTileN);
      const uint32_t empty_off = smem_u32(empty), accf_off = smem_u32(acc_full);
      uint32_t stage = 0, phase = 0, acc_phase = 0, region = 0;
      bool ok = true;
      for (int t = cluster; ok && t < p.num_tiles; t += num_clusters) {
        if (!mbar_wait_cluster(acc_empty, acc_phase ^ 1u, p.status, kStatusTimeoutAccEmpty, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        for (int kt = 0; kt < k_iters; ++kt) {
          if (!mbar_wait_cluster(&ready[stage], phase, p.status, kStatusTimeoutFull, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const int nkb = min(kPairKBlocks, p.sf_kblocks - kPairKBlocks * kt);
          const uint64_t da = sdesc_kmajor_sw128(smem_u32(smem + kPairOffA + stage * kPairABytes));
          const uint64_t db = sdesc_kmajor_sw128(smem_u32(smem + kPairOffB + stage * kPairBBytes));
          const uint32_t tsfa = tmem + kPairSfaCol + region * kPairSfColsPerStage;
          const uint32_t tsfb = tsfa + 4 * kPairKBlocks;
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
          tc_commit_pair_mc(empty_off + 8u * stage, 0xF);  // stage s free in all four CTAs
          if (++stage == kPairStages) {
            stage = 0;
            phase ^= 1u;
          }
          if (++region == kPairSfRegions) region = 0;
        }
        if (!ok) break;
        tc_commit_pair_mc(accf_off, pair_mask);
        acc_phase ^= 1u;
      }
      if (!ok) {
        tc_commit_pair(smem_u32(&drain[0]));
        mbar_wait(&drain[0], 0, p.status, kStatusTimeoutDrain, nullptr);
      }
    }
    __syncwarp();
  } else if (warp == 3 && !leader) {
    // ------------------------------------------------------------------ pair relay (non-leader)
    // This CTA's whole stage (own atom, pushed atom, B) has landed: tell the leader's MMA thread.
    if (lane == 0) {
      uint32_t stage = 0, phase = 0;
      bool ok = true;
      for (int t = cluster; ok && t < p.num_tiles; t += num_clusters) {
        for (int kt = 0; kt < k_iters; ++kt) {
          if (!mbar_wait(&own[stage], phase, p.status, kStatusTimeoutFull, abort_flag) ||
              !mbar_wait(&full[stage], phase, p.status, kStatusTimeoutFull, abort_flag)) {
            ok = false;
            break;
          }
          mbar_arrive_cluster(ready_lead + 8u * stage);
          if (++stage == kPairStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    }
    __syncwarp();
  } else if (warp == 3 || warp == 4 || warp == 9) {
    // ------------------------------------------------------------------ scale copies (pair leaders)
    if (leader && lane == 0) {
      const bool is_a = warp == 3;
      const int half = warp == 9 ? 1 : 0;
      const int role = is_a ? 1 : 2 + half;
      const uint32_t sfe_off = smem_u32(sf_empty);
      uint32_t stage = 0, phase = 0, slot = 0, sphase = 0, region = 0;
      uint32_t lag_stage = 0, lag_phase = 0;
      int it = 0;
      bool ok = true;
      for (int t = cluster; ok && t < p.num_tiles; t += num_clusters) {
        for (int kt = 0; kt < k_iters; ++kt, ++it) {
          if (!mbar_wait(&sf_full[slot], sphase, p.status, kStatusTimeoutFull, abort_flag)) {
            ok = false;
            break;
          }
          if (it >= kPairSfRegions) {
            // TMEM region reuse: the MMAs of iteration it - R have completed (their stage's
            // empty barrier; its count of 2 also waits for the other pair, which only delays).
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
          tc_fence_before();
          if (is_a && (!mbar_wait(&own[stage], phase, p.status, kStatusTimeoutFull, abort_flag) ||
                       !mbar_wait(&full[stage], phase, p.status, kStatusTimeoutFull, abort_flag))) {
            ok = false;
            break;
          }
          mbar_arrive(&ready[stage]);
          tc_commit_pair_mc(sfe_off + 8u * slot, pair_mask);
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
  } else if (warp >= 5 && warp <= 8) {
    // ------------------------------------------------------------------ epilogue (every CTA)
    const int quad = warp & 3;
    const int row = quad * 32 + lane;
    const uint32_t tmem_row = tmem + (static_cast<uint32_t>(quad * 32) << 16);
    const float alpha = *p.alpha;
    const bool evict_first = p.store_evict_first != 0;
    uint32_t acc_phase = 0;
    for (int t = cluster; t < p.num_tiles; t += num_clusters) {
      int mt, ntp;
      quad_tile_coord(p, t, mt, ntp);
      const int nt = 2 * ntp + static_cast<int>(pid);
      if (!mbar_wait(acc_full, acc_phase, p.status, kStatusTimeoutAccFull, abort_flag)) break;
      acc_phase ^= 1u;
      tc_fence_after();
      uint32_t out[kPairTileN / 2];
#pragma unroll
      for (int ch = 0; ch < kPairTileN / 32; ch += 2) {
        uint32_t r0[32], r1[32];
        tmem_ld_32x32b_x32(tmem_row + kAccCol + ch * 32, r0);
        tmem_ld_32x32b_x32(tmem_row + kAccCol + ch * 32 + 32, r1);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          out[ch * 16 + i] = pack_out(__fmul_rn(__uint_as_float(r0[2 * i]), alpha),
                                      __fmul_rn(__uint_as_float(r0[2 * i + 1]), alpha), kBF16);
          out[ch * 16 + 16 + i] = pack_out(__fmul_rn(__uint_as_float(r1[2 * i]), alpha),
                                           __fmul_rn(__uint_as_float(r1[2 * i + 1]), alpha), kBF16);
        }
      }
      tc_fence_before();
      mbar_arrive_cluster(acc_empty_lead);

      const int gm = mt * kPairTileM + 128 * static_cast<int>(prank) + row;
      const int cols_left = p.n - nt * kPairTileN;  // <= 0 for the absent last tile of an odd count
      if (gm < p.m && cols_left > 0) {
        const size_t off = (static_cast<size_t>(gm) * p.ldc + p.col0 + static_cast<size_t>(nt) * kPairTileN) * 2;
        uint8_t* rowp = reinterpret_cast<uint8_t*>(p.c) + off;
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
      if (p.n_peer > 0 && cols_left > 0) {
        __threadfence_block();
        __syncwarp();
        const int row0 = mt * kPairTileM + 128 * static_cast<int>(prank) + quad * 32;
        if (row0 < p.m)
          copy_rows_to_peers(p, row0, min(kPairTileN, cols_left),
                             (static_cast<size_t>(row0) * p.ldc + p.col0 + static_cast<size_t>(nt) * kPairTileN) * 2,
                             lane);
      }
    }
  }

  if (p.n_peer > 0) __threadfence_system();
  tc_fence_before();
  cluster_sync();  // no CTA leaves while another may still push into it or signal its barriers
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, kTmemCols);
  }
}

}  // namespace g3
