// dW2 = grad_y^T . h with h = left * silu(gate) recomputed from preact in the
// GEMM's operand prologue (swiglu_recompute.py:71-73;
// fused_forward_packed.py:310-311), on tcgen05.
//
// The kernel computes dW2^T tiles, D[hidden j, out d] = sum_t h[t, j] grad_y[t, d]:
//   A = h^T  [128 hidden units x K tokens]  built in shared memory by the
//            transform warps from the TMA-loaded left and gate tiles
//   B = grad_y [K tokens x 512 outputs]     TMA-loaded, two N=256 MMAs
//   D        128 TMEM lanes x 512 columns (the whole TMEM, one accumulator)
// so each h element is recomputed Dout/512 times (7 at Dout=3584) instead of
// once per 128-row output tile, and the element-wise work stays well below
// the tensor core's consumption rate. The epilogue writes D transposed into
// dW2 [Dout, H]: lane j holds hidden unit j, so each warp store covers 32
// consecutive hidden units of one output row (64 contiguous bytes).
//
// Warps: 0 TMA producer, 1 TMEM alloc + MMA issuer, 2..5 epilogue,
// 6.. h prologue. Every wait is bounded (see ptx.cuh).
#pragma once

#include "tc_gemm.cuh"

namespace swiglu {

struct Dw2Params {
  CUtensorMap tm_pre;  // preact [M, 2H], box {64 cols, BK tokens}
  CUtensorMap tm_gy;   // grad_y [M, Dout], box {64 outs, BK tokens}
  // CTA-pair kernel, where the shapes allow (`gather` bits): one TMA
  // operation per stage for all four left/gate boxes (bit 0; map {64 cols,
  // tokens, 64-col blocks, left/gate}) and one for all four grad_y boxes
  // (bit 1; map {64 outs, tokens, 64-col blocks, 256-col halves}), in the
  // same shared-memory layout as the four 2-D boxes each replaces.
  CUtensorMap tm_lg4;
  CUtensorMap tm_gy4;
  int gather;
  // dW2 [Dout, H] in {32 units x 32 outputs} boxes, 64-byte swizzle: the
  // CTA-pair kernel's epilogue stores through shared memory and TMA.
  CUtensorMap tm_out;
  __nv_bfloat16* dw2;  // [Dout, H]
  int M, H, Dout;
  int layout;
  int tiles_j, tiles_d;  // hidden blocks of 128, output blocks of 512
  uint32_t* status;
  // Stream-K tail of the pair kernel, as in TcParams (partials [tail][split][256][512]).
  float* sk_partials;
  uint32_t* sk_counters;
  int sk_tail, sk_split;
  uint32_t sk_epoch;
};

struct Dw2Cfg {
  static constexpr int BJ = 128;  // hidden units per tile (UMMA M)
  static constexpr int BD = 512;  // outputs per tile (two UMMA N=256)
  static constexpr int BK = 32;   // tokens per stage
  static constexpr int BOX_BYTES = 64 * BK * 2;     // one {64, BK} bf16 box
  static constexpr int A_BYTES = BJ * BK * 2;       // h^T (left, transformed in place)
  static constexpr int G_BYTES = BJ * BK * 2;       // gate
  static constexpr int B_BYTES = BD * BK * 2;       // grad_y
  static constexpr int STAGE_BYTES = A_BYTES + G_BYTES + B_BYTES;
  static constexpr int STAGES = 4;
  static constexpr int NUM_XFORM_WARPS = 4;
  static constexpr int NUM_THREADS = 32 * (2 + 4 + NUM_XFORM_WARPS);
  static constexpr int TMEM_COLS = 512;
  static constexpr int SMEM_BYTES = 1024 + STAGES * STAGE_BYTES + 8 * (3 * STAGES + 3) + 16;
  static_assert(SMEM_BYTES <= 227 * 1024, "shared memory budget");
};

__global__ void __launch_bounds__(Dw2Cfg::NUM_THREADS, 1) dw2_hprologue_kernel(const __grid_constant__ Dw2Params p) {
  using C = Dw2Cfg;
  constexpr int STAGES = C::STAGES, BK = C::BK;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + STAGES * C::STAGE_BYTES);
  uint64_t* full = bars;                // TMA -> transform
  uint64_t* ready = bars + STAGES;      // transform -> MMA
  uint64_t* empty = bars + 2 * STAGES;  // MMA -> TMA
  uint64_t* tmem_full = bars + 3 * STAGES;
  uint64_t* tmem_empty = tmem_full + 1;
  uint64_t* mma_done = tmem_empty + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const uint32_t warp = warp_id(), lane = lane_id();
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&ready[s], C::NUM_XFORM_WARPS);
      mbar_init(&empty[s], 1);
    }
    mbar_init(tmem_full, 1);
    mbar_init(tmem_empty, 4);
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before_sync();
  __syncthreads();
  tc_fence_after_sync();
  const uint32_t tmem_base = *tmem_slot;
  const int num_tiles = p.tiles_j * p.tiles_d;
  const int num_kb = (p.M + BK - 1) / BK;
  uint32_t* status = p.status;

  // Tiles are visited output-block fastest: CTAs running together share the
  // same hidden block's left/gate rows and stream the same grad_y rows.
  auto tile_jd = [&](int tile, int& tj, int& td) {
    tj = tile / p.tiles_d;
    td = tile - tj * p.tiles_d;
  };

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&p.tm_pre);
      tma_prefetch_desc(&p.tm_gy);
      uint32_t stage = 0, phase = 0, filled = 0, fill_parity = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        int tj, td;
        tile_jd(tile, tj, td);
        const int j0 = tj * C::BJ;
        const int lc = left_col(j0, p.H, p.layout);
        const int gc = gate_col(j0, p.H, p.layout);
        const int d0 = td * C::BD;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag, status, kErrTimeoutProducer)) {
            ok = false;
            break;
          }
          uint8_t* sa = smem + stage * C::STAGE_BYTES;
          uint8_t* sg = sa + C::A_BYTES;
          uint8_t* sb = sg + C::G_BYTES;
          const int t0 = kb * BK;
          mbar_arrive_expect_tx(&full[stage], C::STAGE_BYTES);
          tma_load_2d(sa, &p.tm_pre, &full[stage], lc, t0);
          tma_load_2d(sa + C::BOX_BYTES, &p.tm_pre, &full[stage], lc + 64, t0);
          tma_load_2d(sg, &p.tm_pre, &full[stage], gc, t0);
          tma_load_2d(sg + C::BOX_BYTES, &p.tm_pre, &full[stage], gc + 64, t0);
#pragma unroll
          for (int i = 0; i < C::BD / 64; ++i) tma_load_2d(sb + i * C::BOX_BYTES, &p.tm_gy, &full[stage], d0 + 64 * i, t0);
          filled |= 1u << stage;
          fill_parity = (fill_parity & ~(1u << stage)) | (phase << stage);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      for (int s = 0; s < STAGES; ++s) {
        if (filled & (1u << s)) {
          volatile int never = 0;
          mbar_wait(&full[s], (fill_parity >> s) & 1u, &never, status, kErrTimeoutTeardown);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc_f16(128, 256, 1, 1, 1, 1);  // both operands MN-major
      uint32_t stage = 0, phase = 0, acc_phase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        if (!mbar_wait(tmem_empty, acc_phase ^ 1, abort_flag, status, kErrTimeoutMma)) break;
        tc_fence_after_sync();
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&ready[stage], phase, abort_flag, status, kErrTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after_sync();
          const uint32_t sa = smem_u32(smem + stage * C::STAGE_BYTES);
          const uint32_t sb = sa + C::A_BYTES + C::G_BYTES;
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            const uint64_t adesc = make_smem_desc_sw128(sa + k * 2048, C::BOX_BYTES, 1024);
            const uint64_t b0 = make_smem_desc_sw128(sb + k * 2048, C::BOX_BYTES, 1024);
            const uint64_t b1 = make_smem_desc_sw128(sb + 4 * C::BOX_BYTES + k * 2048, C::BOX_BYTES, 1024);
            const uint32_t acc = (kb | k) != 0 ? 1u : 0u;
            umma_f16_ss(tmem_base, adesc, b0, idesc, acc);
            umma_f16_ss(tmem_base + 256, adesc, b1, idesc, acc);
          }
          umma_commit(&empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        umma_commit(tmem_full);
        acc_phase ^= 1;
      }
      umma_commit(mma_done);
      volatile int never = 0;
      mbar_wait(mma_done, 0, &never, status, kErrTimeoutTeardown);
    }
  } else if (warp < 6) {
    // Epilogue: lane = hidden unit, 32 consecutive outputs per TMEM load.
    const uint32_t q = warp & 3u;
    uint32_t acc_phase = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
      int tj, td;
      tile_jd(tile, tj, td);
      if (!mbar_wait(tmem_full, acc_phase, abort_flag, status, kErrTimeoutEpilogue)) break;
      tc_fence_after_sync();
      const int j = tj * C::BJ + static_cast<int>(q * 32 + lane);
      const bool j_ok = j < p.H;
      const int d0 = td * C::BD;
      const uint32_t t_row = tmem_base + ((q * 32u) << 16);
#pragma unroll 1
      for (int c = 0; c < C::BD / 32; ++c) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(t_row + c * 32, r);
        tmem_ld_wait();
        const int dc = d0 + c * 32;
        if (j_ok) {
          __nv_bfloat16* col = p.dw2 + static_cast<long long>(dc) * p.H + j;
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            if (dc + i < p.Dout) col[static_cast<long long>(i) * p.H] = __float2bfloat16_rn(__uint_as_float(r[i]));
          }
        }
      }
      tc_fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(tmem_empty);
      acc_phase ^= 1;
    }
  } else {
    // h prologue: A (left) and G (gate) were loaded with the same boxes, so
    // h = left * silu(gate) is formed at matching swizzled positions.
    const uint32_t xt = threadIdx.x - 32 * 6;
    constexpr int kChunks = C::A_BYTES / 16;
    uint32_t stage = 0, phase = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
      for (int kb = 0; kb < num_kb; ++kb) {
        if (!mbar_wait(&full[stage], phase, abort_flag, status, kErrTimeoutTransform)) {
          ok = false;
          break;
        }
        uint4* sa = reinterpret_cast<uint4*>(smem + stage * C::STAGE_BYTES);
        const uint4* sg = reinterpret_cast<const uint4*>(smem + stage * C::STAGE_BYTES + C::A_BYTES);
#pragma unroll
        for (int i = static_cast<int>(xt); i < kChunks; i += 32 * C::NUM_XFORM_WARPS) {
          const uint4 lu = sa[i];
          const uint4 gu = sg[i];
          const uint32_t lw[4] = {lu.x, lu.y, lu.z, lu.w};
          const uint32_t gw[4] = {gu.x, gu.y, gu.z, gu.w};
          uint32_t hw[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) hw[e] = swiglu_bf16x2_tanh(lw[e], gw[e]);
          sa[i] = make_uint4(hw[0], hw[1], hw[2], hw[3]);
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&ready[stage]);
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1;
        }
      }
    }
  }

  tc_fence_before_sync();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after_sync();
    tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
}


// ---------------------------------------------------------------------------
// CTA-pair (cta_group::2) version. A pair tile is 256 hidden units x 512
// outputs: rank r recomputes h for its hidden units [128r, 128r+128) only and
// holds 128 of the 256 output columns of each of the two N=256 MMAs, so per
// SM a 48-token stage is 12 KB left + 12 KB gate + 24 KB grad_y and four
// stages fit beside the epilogue's staging. Barriers:
//   lg_full[s]  local, left/gate landed (own TMA)        -> own h prologue
//   b_full[s]   rank 0, both CTAs' grad_y halves landed  -> MMA
//   ready[s]    rank 0, 8 prologue warps finished h      -> MMA
//   empty[s]    each CTA, MMA finished with the stage    -> own producer
//   tmem_full   each CTA; tmem_empty rank 0 (8 epilogue warps)
// ---------------------------------------------------------------------------
struct Dw2PairCfg {
  static constexpr int BJ = 256;   // hidden units per pair tile (UMMA M)
  static constexpr int BJH = 128;  // per CTA
  static constexpr int BD = 512;   // outputs per tile (two UMMA N=256)
  // Tokens per stage. 48 tokens in 4 stages against 32 in 6 (the same bytes
  // in flight, a third fewer stage handshakes) measured 1.048 -> 0.978 ms at
  // M=11136 H=14336 Dout=3584; 64 tokens in 3 stages 0.989 ms.
  static constexpr int BK = 48;
  static constexpr int BOX_BYTES = 64 * BK * 2;
  static constexpr int A_BYTES = BJH * BK * 2;        // left -> h
  static constexpr int G_BYTES = BJH * BK * 2;        // gate
  static constexpr int B_BYTES = (BD / 2) * BK * 2;   // this CTA's grad_y columns
  static constexpr int STAGE_BYTES = A_BYTES + G_BYTES + B_BYTES;
  static constexpr int STAGES = 4;
  // Prologue warps in groups, each group on its own ring slots; measured at
  // M=11136 H=14336 Dout=3584: 4 warps on every stage 1.66 ms, 8 warps on
  // every stage 1.33 ms, 2 groups of 4 warps 1.30 ms.
  static constexpr int NUM_XFORM_WARPS = 8;
  static constexpr int XFORM_GROUPS = 2;
  static constexpr int XFORM_THREADS_PER_GROUP = 32 * NUM_XFORM_WARPS / XFORM_GROUPS;
  static_assert(STAGES % XFORM_GROUPS == 0, "each ring slot must belong to one prologue group");
  static_assert(NUM_XFORM_WARPS % XFORM_GROUPS == 0, "equal prologue groups");
  static constexpr int NUM_THREADS = 32 * (2 + 4 + NUM_XFORM_WARPS);
  static constexpr int TMEM_COLS = 512;
  // Epilogue staging after the ring and its barriers: per epilogue warp two
  // {32 x 32} bf16 boxes (2 KB each) for the transposed TMA stores.
  static constexpr int BAR_BYTES = 8 * (4 * STAGES + 3) + 16;
  static constexpr int EPI_BOX_BYTES = 32 * 64;
  static constexpr int EPI_OFFSET = STAGES * STAGE_BYTES + ((BAR_BYTES + 1023) / 1024) * 1024;
  static constexpr int SMEM_BYTES = 1024 + EPI_OFFSET + 4 * 2 * EPI_BOX_BYTES;
  static_assert(SMEM_BYTES <= 227 * 1024, "shared memory budget");
};

__global__ void __launch_bounds__(Dw2PairCfg::NUM_THREADS, 1)
    dw2_hprologue_pair_kernel(const __grid_constant__ Dw2Params p) {
  using C = Dw2PairCfg;
  constexpr int STAGES = C::STAGES, BK = C::BK;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + STAGES * C::STAGE_BYTES);
  uint64_t* lg_full = bars;
  uint64_t* b_full = bars + STAGES;
  uint64_t* ready = bars + 2 * STAGES;
  uint64_t* empty = bars + 3 * STAGES;
  uint64_t* tmem_full = bars + 4 * STAGES;
  uint64_t* tmem_empty = tmem_full + 1;
  uint64_t* mma_done = tmem_empty + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const uint32_t warp = warp_id(), lane = lane_id();
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&lg_full[s], 1);
      mbar_init(&b_full[s], 1);
      mbar_init(&ready[s], 2 * (C::NUM_XFORM_WARPS / C::XFORM_GROUPS));
      mbar_init(&empty[s], 1);
    }
    mbar_init(tmem_full, 1);
    mbar_init(tmem_empty, 8);
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, C::TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before_sync();
  cluster_sync_all();
  tc_fence_after_sync();
  const uint32_t tmem_base = *tmem_slot;
  const int num_tiles = p.tiles_j * p.tiles_d;
  const int num_units = sk_units(num_tiles, p.sk_tail, p.sk_split);
  const int num_kb = (p.M + BK - 1) / BK;
  const int first_unit = static_cast<int>(cluster_id_x());
  const int unit_step = static_cast<int>(num_clusters_x());
  uint32_t* status = p.status;
  auto tile_jd = [&](int tile, int& tj, int& td) {
    tj = tile / p.tiles_d;
    td = tile - tj * p.tiles_d;
  };

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&p.tm_pre);
      tma_prefetch_desc(&p.tm_gy);
      if (p.gather & 1) tma_prefetch_desc(&p.tm_lg4);
      if (p.gather & 2) tma_prefetch_desc(&p.tm_gy4);
      uint32_t stage = 0, phase = 0, filled = 0, fill_parity = 0;
      bool ok = true;
      for (int u = first_unit; u < num_units && ok; u += unit_step) {
        const SkUnit w = sk_unit_of(num_tiles, p.sk_tail, p.sk_split, u, num_kb);
        int tj, td;
        tile_jd(w.tile, tj, td);
        const int j0 = tj * C::BJ + C::BJH * static_cast<int>(rank);
        const int lc = left_col(j0, p.H, p.layout);
        const int gc = gate_col(j0, p.H, p.layout);
        const int d0 = td * C::BD + 128 * static_cast<int>(rank);
        for (int kb = w.kb0; kb < w.kb1; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag, status, kErrTimeoutProducer)) {
            ok = false;
            break;
          }
          uint8_t* sa = smem + stage * C::STAGE_BYTES;
          uint8_t* sg = sa + C::A_BYTES;
          uint8_t* sb = sg + C::G_BYTES;
          const int t0 = kb * BK;
          mbar_arrive_expect_tx(&lg_full[stage], C::A_BYTES + C::G_BYTES);
          if (p.gather & 1) {
            tma_load_4d(sa, &p.tm_lg4, &lg_full[stage], 0, t0, lc / 64, 0);
          } else {
            tma_load_2d(sa, &p.tm_pre, &lg_full[stage], lc, t0);
            tma_load_2d(sa + C::BOX_BYTES, &p.tm_pre, &lg_full[stage], lc + 64, t0);
            tma_load_2d(sg, &p.tm_pre, &lg_full[stage], gc, t0);
            tma_load_2d(sg + C::BOX_BYTES, &p.tm_pre, &lg_full[stage], gc + 64, t0);
          }
          const uint32_t bbar = map_to_rank(&b_full[stage], 0);
          if (leader) mbar_arrive_expect_tx(&b_full[stage], 2 * C::B_BYTES);
          if (p.gather & 2) {
            tma_load_4d_pair(sb, &p.tm_gy4, bbar, 0, t0, d0 / 64, 0);
          } else {
            tma_load_2d_pair(sb, &p.tm_gy, bbar, d0, t0);
            tma_load_2d_pair(sb + C::BOX_BYTES, &p.tm_gy, bbar, d0 + 64, t0);
            tma_load_2d_pair(sb + 2 * C::BOX_BYTES, &p.tm_gy, bbar, d0 + 256, t0);
            tma_load_2d_pair(sb + 3 * C::BOX_BYTES, &p.tm_gy, bbar, d0 + 320, t0);
          }
          filled |= 1u << stage;
          fill_parity = (fill_parity & ~(1u << stage)) | (phase << stage);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      for (int s = 0; s < STAGES; ++s) {
        if (filled & (1u << s)) {
          volatile int never = 0;
          mbar_wait(&empty[s], (fill_parity >> s) & 1u, &never, status, kErrTimeoutTeardown);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      constexpr uint32_t idesc = make_idesc_f16(256, 256, 1, 1, 1, 1);
      uint32_t stage = 0, phase = 0, acc_phase = 0;
      bool ok = true;
      for (int u = first_unit; u < num_units && ok; u += unit_step) {
        const SkUnit w = sk_unit_of(num_tiles, p.sk_tail, p.sk_split, u, num_kb);
        if (!mbar_wait(tmem_empty, acc_phase ^ 1, abort_flag, status, kErrTimeoutMma)) break;
        tc_fence_after_sync();
        for (int kb = w.kb0; kb < w.kb1; ++kb) {
          if (!mbar_wait(&b_full[stage], phase, abort_flag, status, kErrTimeoutMma) ||
              !mbar_wait(&ready[stage], phase, abort_flag, status, kErrTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after_sync();
          const uint32_t sa = smem_u32(smem + stage * C::STAGE_BYTES);
          const uint32_t sb = sa + C::A_BYTES + C::G_BYTES;
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            const uint64_t adesc = make_smem_desc_sw128(sa + k * 2048, C::BOX_BYTES, 1024);
            const uint64_t b0 = make_smem_desc_sw128(sb + k * 2048, C::BOX_BYTES, 1024);
            const uint64_t b1 = make_smem_desc_sw128(sb + 2 * C::BOX_BYTES + k * 2048, C::BOX_BYTES, 1024);
            const uint32_t acc = (kb != w.kb0 || k != 0) ? 1u : 0u;
            umma_f16_ss_pair(tmem_base, adesc, b0, idesc, acc);
            umma_f16_ss_pair(tmem_base + 256, adesc, b1, idesc, acc);
          }
          umma_commit_pair(map_to_rank(&empty[stage], 0));
          umma_commit_pair(map_to_rank(&empty[stage], 1));
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        umma_commit_pair(map_to_rank(tmem_full, 0));
        umma_commit_pair(map_to_rank(tmem_full, 1));
        acc_phase ^= 1;
      }
      umma_commit_pair(map_to_rank(mma_done, 0));
      volatile int never = 0;
      mbar_wait(mma_done, 0, &never, status, kErrTimeoutTeardown);
    }
  } else if (warp < 6) {
    const uint32_t q = warp & 3u;
    uint32_t acc_phase = 0;
    for (int u = first_unit; u < num_units; u += unit_step) {
      const SkUnit w = sk_unit_of(num_tiles, p.sk_tail, p.sk_split, u, num_kb);
      int tj, td;
      tile_jd(w.tile, tj, td);
      if (!mbar_wait(tmem_full, acc_phase, abort_flag, status, kErrTimeoutEpilogue)) break;
      tc_fence_after_sync();
      const int j_in_tile = C::BJH * static_cast<int>(rank) + static_cast<int>(q * 32 + lane);
      const int jw = tj * C::BJ + C::BJH * static_cast<int>(rank) + static_cast<int>(q * 32);  // warp's first unit
      const int d0 = td * C::BD;
      const uint32_t t_row = tmem_base + ((q * 32u) << 16);
      bool finish = true;
      if (w.parts > 1) {
        // Stream-K part: the last of the parts to arrive for this 32-row
        // slab finishes the tile.
        const int i = w.tile - (num_tiles - p.sk_tail);
        const long long part_stride = static_cast<long long>(C::BJ) * C::BD;
        const float* fix = p.sk_partials + (static_cast<long long>(i) * w.parts * C::BJ + j_in_tile) * C::BD;
        finish = sk_publish_and_fix(t_row, C::BD, const_cast<float*>(fix) + w.part * part_stride, fix, part_stride,
                                    w.parts, p.sk_counters + i * 8 + rank * 4 + q, p.sk_epoch);
      }
      // D is hidden-major (lane = unit) and dW2 output-major: each 32-output
      // chunk is transposed into a {32 units x 32 outputs} box (row i =
      // output dc + i, 64-byte rows, 64-byte swizzle: 16-byte chunk k of row
      // i at k ^ ((i >> 1) & 3)) and leaves with one TMA store, which skips
      // the parts of the box beyond H or Dout.
      uint8_t* ebuf = smem + C::EPI_OFFSET + q * 2 * C::EPI_BOX_BYTES;
#pragma unroll 1
      for (int c = 0; c < (finish ? C::BD / 32 : 0); ++c) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(t_row + c * 32, r);
        tmem_ld_wait();
        const int dc = d0 + c * 32;
        uint8_t* buf = ebuf + (c & 1) * C::EPI_BOX_BYTES;
        // The store issued from this buffer two chunks ago (possibly in the
        // previous tile) has read it once at most one store is still reading.
        if (lane == 0) bulk_wait_read<1>();
        __syncwarp();
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const uint32_t off = i * 64 + ((((lane >> 3) ^ ((i >> 1) & 3u))) << 4) + (lane & 7u) * 2;
          *reinterpret_cast<__nv_bfloat16*>(buf + off) = __float2bfloat16_rn(__uint_as_float(r[i]));
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0 && jw < p.H && dc < p.Dout) {
          tma_store_2d(&p.tm_out, buf, jw, dc);
          bulk_commit();
        }
      }
      tc_fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(map_to_rank(tmem_empty, 0));
      acc_phase ^= 1;
    }
    // The TMA stores read shared memory asynchronously: finish before exit.
    if (lane == 0) bulk_wait_read<0>();
  } else {
    // The prologue warps form C::XFORM_GROUPS groups and ring slot s belongs
    // to group s % G (G divides STAGES), so G stages are transformed
    // concurrently (per-stage latency, not the math rate, limits a single
    // stage in flight). Owning whole slots keeps the parity protocol exact: a
    // group waits on every phase of its slots in order, so a parity test can
    // never match a phase two generations old.
    const uint32_t xw = threadIdx.x - 32 * 6;
    const uint32_t grp = xw / C::XFORM_THREADS_PER_GROUP;
    const uint32_t xt = xw % C::XFORM_THREADS_PER_GROUP;
    constexpr int kChunks = C::A_BYTES / 16;
    uint32_t stage = 0, phase = 0;
    bool ok = true;
    for (int u = first_unit; u < num_units && ok; u += unit_step) {
      const SkUnit w = sk_unit_of(num_tiles, p.sk_tail, p.sk_split, u, num_kb);
      for (int kb = w.kb0; kb < w.kb1; ++kb) {
        if (stage % C::XFORM_GROUPS == grp) {
          if (!mbar_wait(&lg_full[stage], phase, abort_flag, status, kErrTimeoutTransform)) {
            ok = false;
            break;
          }
          uint4* sa = reinterpret_cast<uint4*>(smem + stage * C::STAGE_BYTES);
          const uint4* sg = reinterpret_cast<const uint4*>(smem + stage * C::STAGE_BYTES + C::A_BYTES);
#pragma unroll
          for (int i = static_cast<int>(xt); i < kChunks; i += C::XFORM_THREADS_PER_GROUP) {
            const uint4 lu = sa[i];
            const uint4 gu = sg[i];
            const uint32_t lw[4] = {lu.x, lu.y, lu.z, lu.w};
            const uint32_t gw[4] = {gu.x, gu.y, gu.z, gu.w};
            uint32_t hw[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) hw[e] = swiglu_bf16x2_tanh(lw[e], gw[e]);
            sa[i] = make_uint4(hw[0], hw[1], hw[2], hw[3]);
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) mbar_arrive_cluster(map_to_rank(&ready[stage], 0));
        }
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1;
        }
      }
    }
  }

  tc_fence_before_sync();
  __syncthreads();
  cluster_sync_all();
  if (warp == 1) {
    tc_fence_after_sync();
    tmem_dealloc_pair(tmem_base, C::TMEM_COLS);
  }
}

}  // namespace swiglu
