// 2-SM (cta_group::2) variant of the persistent warp-specialized GEMM.
//
// A cluster of two CTAs on neighbouring SMs computes one 256 x (256·NSUB)
// output tile with M=256, N=256 tcgen05.mma instructions issued by rank 0
// (NSUB of them per 16-deep k-step). Each CTA stages only its half of the
// operands (A rows [128r, 128r+128) and, of each MMA's 256 B columns, the
// 128 at [128r, 128r+128)) and its TMEM receives its 128 rows of D, so per
// SM the shared-memory footprint per MMA-clock and the L2 operand traffic are
// half those of the single-SM kernel (tc_gemm.cuh); with NSUB = 2 a further
// quarter less (see Tc2Cfg).
//
// Protocol (all waits bounded):
//   both CTAs' producers wait on their own `empty[s]` and TMA-load their halves
//     with completion counted on rank 0's `full[s]` (rank 0 posts the
//     expected byte count of both halves);
//   rank 0's MMA thread waits `full[s]`, issues the pair MMAs and commits to
//     `empty[s]` of both CTAs, and per tile to `tmem_full[acc]` of both CTAs;
//   both CTAs' epilogue warps drain their TMEM rows and arrive on rank 0's
//     `tmem_empty[acc]` (8 arrivals: 4 warps x 2 CTAs); with NSUB = 2 the
//     single accumulator's two 256-column halves are freed one by one
//     (`tmem_empty[0]`, `[1]`) and the MMA thread starts the next tile on
//     half 0 while half 1 drains.
// Epilogues: each 256-column half is written as a tile of its own; plain
// stores, SwiGLU (kEpiSwigluTma) and dSwiGLU go through swizzled shared-memory
// boxes and TMA (tc_gemm.cuh), the rest through epilogue_tile.
//
// No TMA multicast is used: each CTA loads its own halves.
#pragma once

#include "tc_gemm.cuh"

namespace swiglu {

// NSUB = N=256 MMAs per k-step: 1 gives 256 x 256 pair tiles with the
// accumulator double-buffered in TMEM (the epilogue of one tile overlaps the
// next tile's main loop); 2 gives 256 x 512 pair tiles whose single
// accumulator fills the CTA's 512 TMEM columns: per MMA FLOP a CTA then loads
// 25 % fewer operand bytes from L2 (A is shared by both N halves), and the
// epilogue runs between main loops while TMA keeps filling the ring.
template <bool A_MN_, bool B_MN_, int EPI_, bool OUT_F32_, int NSUB_ = 1, bool FP8_ = false>
struct Tc2Cfg {
  static constexpr int NSUB = NSUB_;
  // FP8_: e4m3 operands (kind::f8f6f4), both K-major, rows scaled in the
  // epilogue by scale_a[row] * scale_b[col] (TcParams).
  static constexpr bool FP8 = FP8_;
  static_assert(!FP8_ || (!A_MN_ && !B_MN_), "e4m3 operands are K-major here");
  static_assert(!FP8_ || EPI_ == kEpiStore || EPI_ == kEpiSwigluTma, "scaled epilogues: store and SwiGLU-TMA");
  static_assert(NSUB == 1 || NSUB == 2, "one or two N=256 MMAs per k-step");
  static constexpr int BM = 256;          // pair tile rows (128 per CTA)
  static constexpr int BMH = 128;         // rows per CTA
  static constexpr int BN = 256 * NSUB;   // tile columns (BN / 2 of B per CTA)
  // One 128-byte swizzle row of K per stage: 64 bf16 or 128 e4m3 elements,
  // four MMAs of K = 16 (bf16) or K = 32 (e4m3), 32 bytes each.
  static constexpr int ES = FP8_ ? 1 : 2;
  static constexpr int BK = 128 / ES;
  static constexpr int KSTEPS = 4;
  static constexpr bool A_MN = A_MN_;
  static constexpr bool B_MN = B_MN_;
  static constexpr int EPI = EPI_;
  static constexpr bool OUT_F32 = OUT_F32_;
  static constexpr int A_BYTES = BMH * BK * ES;        // 16 KB
  static constexpr int SUB_B_BYTES = 128 * BK * ES;    // 16 KB: this CTA's half of one N=256 MMA's B
  static constexpr int B_BYTES = NSUB * SUB_B_BYTES;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  // The dSwiGLU epilogue stages preact, grad and h boxes (48 KB), one ring
  // stage's worth of shared memory.
  static constexpr int STAGES = (NSUB == 1 ? 6 : 4) - (EPI_ == kEpiDswiglu ? 1 : 0);
  static constexpr int ACCS = NSUB == 1 ? 2 : 1;       // accumulator buffers in TMEM
  static constexpr int TMEM_COLS = 512;
  static constexpr int NUM_THREADS = 192;
  static constexpr int BAR_BYTES = 8 * (2 * STAGES + 5) + 16;
  static constexpr int EPI_STAGE_OFFSET = STAGES * STAGE_BYTES + ((BAR_BYTES + 1023) / 1024) * 1024;
  static constexpr int EPI_STAGE_BYTES = EPI == kEpiScatterRows ? 4 * kScatterStageFloats * 4
                                         : EPI == kEpiStore     ? 4 * StoreStage<OUT_F32>::kWarpBytes
                                         : EPI == kEpiSwigluTma ? 4 * SwigluStage::kWarpBytes
                                         : EPI == kEpiDswiglu   ? 4 * DswigluStage::kWarpBytes + 64
                                                                : 0;
  static constexpr int SMEM_BYTES = 1024 + EPI_STAGE_OFFSET + EPI_STAGE_BYTES;
  static_assert(SMEM_BYTES <= 227 * 1024, "shared memory budget");
};

template <class Cfg>
__global__ void __launch_bounds__(Cfg::NUM_THREADS, 1) tc_gemm2_kernel(const __grid_constant__ TcParams p) {
  constexpr int BN = Cfg::BN, BK = Cfg::BK, STAGES = Cfg::STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + STAGES * Cfg::STAGE_BYTES);
  uint64_t* full = bars;                    // TMA (both CTAs) -> MMA; used in rank 0
  uint64_t* empty = bars + STAGES;          // MMA -> TMA, in each CTA
  uint64_t* tmem_full = bars + 2 * STAGES;  // MMA -> epilogue, in each CTA (2)
  uint64_t* tmem_empty = tmem_full + 2;     // epilogues -> MMA; used in rank 0 (2)
  uint64_t* mma_done = tmem_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const uint32_t warp = warp_id(), lane = lane_id();
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tmem_full[a], 1);
      mbar_init(&tmem_empty[a], 8);
    }
    mbar_init(mma_done, 1);
    if constexpr (Cfg::EPI == kEpiDswiglu) {
      uint64_t* lb = reinterpret_cast<uint64_t*>(smem + Cfg::EPI_STAGE_OFFSET + 4 * DswigluStage::kWarpBytes);
      for (int i = 0; i < 8; ++i) mbar_init(&lb[i], 1);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, Cfg::TMEM_COLS);
    tmem_relinquish_pair();
  }
  // Both CTAs' barriers exist and TMEM is allocated before any cross-CTA use.
  tc_fence_before_sync();
  cluster_sync_all();
  tc_fence_after_sync();
  const uint32_t tmem_base = *tmem_slot;

  const int num_units = sk_num_units(p);
  const int num_kb = (p.K + BK - 1) / BK;
  const int first_unit = static_cast<int>(cluster_id_x());
  const int unit_step = static_cast<int>(num_clusters_x());
  uint32_t* status = p.status;

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&p.tmA);
      tma_prefetch_desc(&p.tmB);
      uint32_t stage = 0, phase = 0, filled = 0, fill_parity = 0;
      bool ok = true;
      for (int u = first_unit; u < num_units && ok; u += unit_step) {
        const SkUnit w = sk_unit(p, u, num_kb);
        int pm, pn;
        tile_coords(w.tile, p.tiles_m, p.tiles_n, p.group_m, pm, pn);
        const int m0 = pm * Cfg::BM + Cfg::BMH * static_cast<int>(rank);
        // First B column of this CTA's 128-column half of each N=256 MMA.
        int b0[Cfg::NSUB];
#pragma unroll
        for (int sub = 0; sub < Cfg::NSUB; ++sub) {
          if constexpr (is_swiglu(Cfg::EPI)) {
            const int j0 = pn * (BN / 2);  // the tile's BN/2 hidden units start at j0
            // MMA `sub` covers units j0 + 128 sub .. + 127: rank 0 holds their
            // left columns, rank 1 their gate columns, so each 256-column half
            // of the accumulator is [left 128 | gate 128] and drains on its own.
            const int j = j0 + 128 * sub;
            b0[sub] = leader ? left_col(j, p.H, p.layout) : gate_col(j, p.H, p.layout);
          } else {
            b0[sub] = pn * BN + 256 * sub + 128 * static_cast<int>(rank);
          }
        }
        for (int kb = w.kb0; kb < w.kb1; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag, status, kErrTimeoutProducer)) {
            ok = false;
            break;
          }
          uint8_t* sa = smem + stage * Cfg::STAGE_BYTES;
          uint8_t* sb = sa + Cfg::A_BYTES;
          const uint32_t bar = map_to_rank(&full[stage], 0);
          if (leader) mbar_arrive_expect_tx(&full[stage], 2 * Cfg::STAGE_BYTES);
          const int k0 = kb * BK;
          if constexpr (Cfg::A_MN) {
            tma_load_2d_pair(sa, &p.tmA, bar, m0, k0);
            tma_load_2d_pair(sa + 64 * BK * 2, &p.tmA, bar, m0 + 64, k0);
          } else {
            tma_load_2d_pair(sa, &p.tmA, bar, k0, m0);
          }
#pragma unroll
          for (int sub = 0; sub < Cfg::NSUB; ++sub) {
            uint8_t* sbs = sb + sub * Cfg::SUB_B_BYTES;
            if constexpr (Cfg::B_MN) {
              tma_load_2d_pair(sbs, &p.tmB, bar, b0[sub], k0);
              tma_load_2d_pair(sbs + 64 * BK * 2, &p.tmB, bar, b0[sub] + 64, k0);
            } else {
              tma_load_2d_pair(sbs, &p.tmB, bar, k0, b0[sub]);
            }
          }
          filled |= 1u << stage;
          fill_parity = (fill_parity & ~(1u << stage)) | (phase << stage);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      // Drain: a stage this CTA filled is finished once the MMA released it.
      for (int s = 0; s < STAGES; ++s) {
        if (filled & (1u << s)) {
          volatile int never = 0;
          mbar_wait(&empty[s], (fill_parity >> s) & 1u, &never, status, kErrTimeoutTeardown);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      constexpr uint32_t idesc = Cfg::FP8 ? make_idesc_e4m3(256, 256)
                                          : make_idesc_f16(256, 256, 1, 1, Cfg::A_MN ? 1 : 0, Cfg::B_MN ? 1 : 0);
      uint32_t stage = 0, phase = 0, acc = 0, acc_phase = 0;
      bool ok = true;
      // The MMAs of one k-block of one 256-column accumulator half.
      auto issue_sub = [&](uint32_t st, int sub, uint32_t d_tmem, bool first_kb) {
        const uint32_t sa = smem_u32(smem + st * Cfg::STAGE_BYTES);
        const uint32_t sbs = sa + Cfg::A_BYTES + sub * Cfg::SUB_B_BYTES;
#pragma unroll
        for (int k = 0; k < Cfg::KSTEPS; ++k) {
          const uint64_t adesc = Cfg::A_MN ? make_smem_desc_sw128(sa + k * 2048, p.mn_lbo, p.mn_sbo)
                                           : make_smem_desc_sw128(sa + k * 32, 16, 1024);
          const uint64_t bdesc = Cfg::B_MN ? make_smem_desc_sw128(sbs + k * 2048, p.mn_lbo, p.mn_sbo)
                                           : make_smem_desc_sw128(sbs + k * 32, 16, 1024);
          if constexpr (Cfg::FP8) {
            umma_f8_ss_pair(d_tmem + 256 * sub, adesc, bdesc, idesc, (!first_kb || k != 0) ? 1u : 0u);
          } else {
            umma_f16_ss_pair(d_tmem + 256 * sub, adesc, bdesc, idesc, (!first_kb || k != 0) ? 1u : 0u);
          }
        }
      };
      auto release = [&](uint32_t st) {
        umma_commit_pair(map_to_rank(&empty[st], 0));
        umma_commit_pair(map_to_rank(&empty[st], 1));
      };
      for (int u = first_unit; u < num_units && ok; u += unit_step) {
        const SkUnit w = sk_unit(p, u, num_kb);
        const uint32_t d_tmem = tmem_base + acc * BN;
        int kb = w.kb0;
        if constexpr (Cfg::NSUB == 2) {
          // One accumulator fills TMEM, but the epilogue frees its halves one
          // after the other (tmem_empty[0], then [1]): start this tile on half
          // 0 for up to a ring's worth of k-blocks while half 1 still drains,
          // then back-fill half 1 for those k-blocks and release their stages.
          // Each half still accumulates its k-blocks in order.
          if (!mbar_wait(&tmem_empty[0], acc_phase ^ 1, abort_flag, status, kErrTimeoutMma)) break;
          tc_fence_after_sync();
          const int ahead = min(STAGES, w.kb1 - w.kb0);
          const uint32_t stage0 = stage;
          for (int i = 0; i < ahead; ++i) {
            if (!mbar_wait(&full[stage], phase, abort_flag, status, kErrTimeoutMma)) {
              ok = false;
              break;
            }
            tc_fence_after_sync();
            issue_sub(stage, 0, d_tmem, i == 0);
            if (++stage == STAGES) {
              stage = 0;
              phase ^= 1;
            }
          }
          if (!ok) break;
          if (!mbar_wait(&tmem_empty[1], acc_phase ^ 1, abort_flag, status, kErrTimeoutMma)) break;
          tc_fence_after_sync();
          for (int i = 0; i < ahead; ++i) {
            const uint32_t st = (stage0 + i) % STAGES;
            issue_sub(st, 1, d_tmem, i == 0);
            release(st);
          }
          kb += ahead;
        } else {
          if (!mbar_wait(&tmem_empty[acc], acc_phase ^ 1, abort_flag, status, kErrTimeoutMma)) break;
          tc_fence_after_sync();
        }
        for (; kb < w.kb1; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort_flag, status, kErrTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after_sync();
#pragma unroll
          for (int sub = 0; sub < Cfg::NSUB; ++sub) issue_sub(stage, sub, d_tmem, kb == w.kb0);
          release(stage);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        umma_commit_pair(map_to_rank(&tmem_full[acc], 0));
        umma_commit_pair(map_to_rank(&tmem_full[acc], 1));
        if (++acc == Cfg::ACCS) {
          acc = 0;
          acc_phase ^= 1;
        }
      }
      umma_commit_pair(map_to_rank(mma_done, 0));
      volatile int never = 0;
      mbar_wait(mma_done, 0, &never, status, kErrTimeoutTeardown);
    }
  } else {
    const uint32_t q = warp & 3u;
    uint32_t acc = 0, acc_phase = 0;
    uint32_t dsw_phase = 0;  // parities of this warp's two preact-load barriers (dSwiGLU)
    uint8_t* dsw_stage = smem + Cfg::EPI_STAGE_OFFSET + (warp - 2) * DswigluStage::kWarpBytes;
    uint64_t* dsw_bar =
        reinterpret_cast<uint64_t*>(smem + Cfg::EPI_STAGE_OFFSET + 4 * DswigluStage::kWarpBytes) + 2 * (warp - 2);
    bool epi_ok = true;
    for (int u = first_unit; u < num_units && epi_ok; u += unit_step) {
      const SkUnit w = sk_unit(p, u, num_kb);
      int pm, pn;
      tile_coords(w.tile, p.tiles_m, p.tiles_n, p.group_m, pm, pn);
      if (!mbar_wait(&tmem_full[acc], acc_phase, abort_flag, status, kErrTimeoutEpilogue)) break;
      tc_fence_after_sync();
      const int row_in_tile = Cfg::BMH * static_cast<int>(rank) + static_cast<int>(q * 32 + lane);
      const int row = pm * Cfg::BM + row_in_tile;
      const uint32_t t_row = tmem_base + ((q * 32u) << 16) + acc * BN;
      float* stage = reinterpret_cast<float*>(smem + Cfg::EPI_STAGE_OFFSET) + (warp - 2) * kScatterStageFloats;
      uint8_t* store_stage = smem + Cfg::EPI_STAGE_OFFSET + (warp - 2) * StoreStage<Cfg::OUT_F32>::kWarpBytes;
      const int row0 = pm * Cfg::BM + Cfg::BMH * static_cast<int>(rank) + static_cast<int>(q * 32);
      uint8_t* swiglu_stage = smem + Cfg::EPI_STAGE_OFFSET + (warp - 2) * SwigluStage::kWarpBytes;
      // Epilogue of accumulator half `sub` (256 columns): a 256-column tile
      // of its own, column block pn * NSUB + sub.
      auto finish_sub = [&](int sub) {
        const int pns = pn * Cfg::NSUB + sub;
        const uint32_t ts = t_row + 256 * sub;
        if constexpr (Cfg::EPI == kEpiStore) {
          epilogue_store_tma<256, Cfg::OUT_F32, Cfg::FP8>(p, pns, row0, ts, store_stage);
        } else if constexpr (Cfg::EPI == kEpiSwigluTma) {
          epilogue_swiglu_tma<256, Cfg::FP8>(p, pns, row0, ts, swiglu_stage);
        } else if constexpr (Cfg::EPI == kEpiDswiglu) {
          // host ensures H % 32 == 0
          epi_ok = epi_ok && epilogue_dswiglu_tma<256>(p, pns, row0, ts, dsw_stage, dsw_bar, dsw_phase, abort_flag);
        } else {
          epilogue_tile<256, Cfg::EPI, Cfg::OUT_F32>(p, pm, pns, row, ts, stage);
        }
      };
      // Frees accumulator half `sub` (NSUB == 2) or the whole buffer.
      auto free_acc = [&](int sub) {
        tc_fence_before_sync();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(map_to_rank(&tmem_empty[Cfg::NSUB == 2 ? sub : acc], 0));
      };
      if (w.parts == 1) {
#pragma unroll 1
        for (int sub = 0; sub < Cfg::NSUB; ++sub) {
          finish_sub(sub);
          free_acc(sub);
        }
      } else {
        // Stream-K part: the last of the parts to arrive for this 32-row
        // slab finishes the tile.
        const int i = w.tile - (p.tiles_m * p.tiles_n - p.sk_tail);
        const long long part_stride = static_cast<long long>(Cfg::BM) * BN;
        const float* fix = p.sk_partials + (static_cast<long long>(i) * w.parts * Cfg::BM + row_in_tile) * BN;
        if (sk_publish_and_fix(t_row, BN, const_cast<float*>(fix) + w.part * part_stride, fix, part_stride, w.parts,
                               p.sk_counters + i * 8 + rank * 4 + q, p.sk_epoch)) {
          for (int sub = 0; sub < Cfg::NSUB; ++sub) finish_sub(sub);
        }
        for (int sub = 0; sub < Cfg::NSUB; ++sub) free_acc(sub);
      }
      if (++acc == Cfg::ACCS) {
        acc = 0;
        acc_phase ^= 1;
      }
    }
    // The TMA stores read shared memory asynchronously: finish before exit.
    if constexpr (Cfg::EPI == kEpiStore || Cfg::EPI == kEpiSwigluTma || Cfg::EPI == kEpiDswiglu) {
      if (lane == 0) bulk_wait_read<0>();
    }
  }

  // Neither CTA releases TMEM (or exits) before the pair is done with it.
  tc_fence_before_sync();
  __syncthreads();
  cluster_sync_all();
  if (warp == 1) {
    tc_fence_after_sync();
    tmem_dealloc_pair(tmem_base, Cfg::TMEM_COLS);
  }
}

}  // namespace swiglu
