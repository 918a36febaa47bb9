// Persistent, warp-specialized tcgen05 GEMM for sm_100a with the SwiGLU
// prologue/epilogue variants of the recompute MLP.
//
//   D[M, N] = A[M, K] * B[K, N]      bf16 operands, f32 accumulation in TMEM
//
// Operands are staged in shared memory by TMA with the 128-byte swizzle and
// consumed by tcgen05.mma straight from shared memory. Each operand may be
// K-major (K contiguous) or MN-major (M resp. N contiguous); the kernel picks
// the TMA box orientation and the UMMA descriptor major-ness accordingly, so
// every transposed GEMM of the backward pass runs without a transpose copy.
//
// Warp roles (one CTA per SM, tiles visited in the grouped order of the
// reference's `_compute_pid`, fused_forward.py:82-94):
//   warp 0      TMA producer (one elected lane)
//   warp 1      TMEM allocator + MMA issuer (one elected lane)
//   warps 2..5  epilogue: TMEM -> registers -> epilogue math -> global
//
// The accumulator is double-buffered in TMEM (2 x BN columns), so the
// epilogue of tile i overlaps the main loop of tile i+1.
//
// Epilogue kinds:
//   kEpiStore    D -> out0 (bf16 or f32)
//   kEpiSwiglu   forward GEMM1: tile columns [0,BN/2) are `left`, [BN/2,BN)
//                `gate` of the same hidden columns; writes preact (left, gate
//                at their standard or packed positions) and h = left*silu(gate)
//                (fused_forward.py:101-185, fused_forward_packed.py:129-183)
//   kEpiDswiglu  backward grad_h GEMM: D = grad_h; reads preact, writes
//                grad_left / grad_gate over it in place
//                (swiglu_recompute.py:33-49, fused_forward_packed.py:222-259)
//                and, if out1 is set, h = left * silu(gate) of the preact it
//                read into out1 [M, H] (swiglu_recompute.py:71), the operand
//                of a plain dW2 GEMM
//   kEpiScatterRows  tensor-parallel: f32 rows pushed into their owner
//                rank's receive buffer (see epilogue_tile)
//   kEpiSwigluTma    kEpiSwiglu storing through shared memory and TMA
//                (2-SM kernel only)
// In the 2-SM kernel (tc_gemm2.cuh) the store, SwiGLU-TMA and dSwiGLU
// epilogues move their tiles as {32 x 32} boxes through swizzled shared
// memory and TMA (epilogue_store_tma, epilogue_swiglu_tma,
// epilogue_dswiglu_tma); the per-lane forms below serve the single-SM kernel
// and the small-M forward.
// The dW2 GEMM with the h prologue is a separate kernel (tc_dw2.cuh).
#pragma once

#include "ptx.cuh"

namespace swiglu {

enum EpiKind : int { kEpiStore = 0, kEpiSwiglu = 1, kEpiDswiglu = 2, kEpiScatterRows = 3, kEpiSwigluTma = 4 };
// kEpiSwigluTma: the SwiGLU epilogue storing through shared memory and TMA
// (2-SM kernel only). A kind of its own so that the per-lane SwiGLU kernel
// does not reserve the staging buffers: shared memory taken from the
// unified L1 slowed that kernel by 10 % at M = 1024.
__host__ __device__ constexpr bool is_swiglu(int epi) { return epi == kEpiSwiglu || epi == kEpiSwigluTma; }
enum Layout : int { kLayoutStd = 0, kLayoutPacked = 1 };

constexpr int kPackChunk = 128;  // BLOCK_SIZE_N_HALF of the packed layout (fused_forward_packed.py:41)

// Column of `left` / `gate` hidden unit j inside a [.., 2H] preact/weight row.
// Standard layout: [left | gate]; packed: [left0|gate0|left1|gate1|...] in
// 128-column chunks (fused_forward_packed.py:77-92).
__host__ __device__ __forceinline__ int left_col(int j, int H, int layout) {
  return layout == kLayoutStd ? j : 2 * (j & ~(kPackChunk - 1)) + (j & (kPackChunk - 1));
}
__host__ __device__ __forceinline__ int gate_col(int j, int H, int layout) {
  return layout == kLayoutStd ? H + j : 2 * (j & ~(kPackChunk - 1)) + kPackChunk + (j & (kPackChunk - 1));
}

struct TcParams {
  CUtensorMap tmA;  // A operand (box: K-major {64,128} / MN-major {64,64})
  CUtensorMap tmB;  // B operand (box: K-major {64,BN/2} / MN-major {64,64})
  CUtensorMap tmC;  // TMA-store epilogues (2-SM kernel), {32 x 32} boxes: store: D; swiglu: preact
  CUtensorMap tmD;  // swiglu TMA-store epilogue: h
  void* out0;       // store: D; swiglu: preact; dswiglu: preact (in/out)
  void* out1;       // swiglu: h (may be null)
  long long ld0, ld1;
  int M, N, K;      // N: output columns (swiglu/dswiglu: hidden units)
  int H;            // hidden width (column maps)
  int layout;       // kLayoutStd / kLayoutPacked
  int tiles_m, tiles_n, group_m;
  int flags;        // kFlagHFromRounded
  uint32_t mn_lbo;  // MN-major operands: byte offset between 64-element MN blocks
  uint32_t mn_sbo;  // MN-major operands: byte offset between 8-row K groups
  uint32_t* status; // device error word
  // kEpiScatterRows: f32 row r of D goes to rank r / rows_per_rank's buffer
  // peer[r / rows_per_rank], at row src_rank * rows_per_rank + r % rows_per_rank
  // (row pitch ld0). The buffers may be other GPUs' memory (NVLink P2P).
  float* peer[8];
  int rows_per_rank, src_rank;
  // e4m3 GEMMs (2-SM kernel): per-row dequantisation factors of A ([M]) and
  // of B's rows ([N]; SwiGLU: indexed by the B row of each left / gate unit).
  const float* scale_a;
  const float* scale_b;
  // Stream-K tail (2-SM kernel only). The last `sk_tail` tiles of the tile
  // order are each computed as `sk_split` parts over equal K ranges by
  // different CTA pairs, so the last round keeps every pair busy. Each part
  // leaves its f32 accumulator tile in `sk_partials` ([tail][split][BM][BN]);
  // per 32-row slab, the warp that arrives last on `sk_counters` (epoch-tagged,
  // see sk_arrive_last) adds the parts in part order and runs the epilogue.
  // sk_split <= 1 disables it (sk_tail is then 0).
  float* sk_partials;
  uint32_t* sk_counters;
  int sk_tail, sk_split;
  uint32_t sk_epoch;  // 1 .. 2^24-1, new for every launch
};

// One unit of stream-K work: tile `tile`, K blocks [kb0, kb1), part `part` of
// `parts` (parts == 1: a whole tile).
struct SkUnit {
  int tile, part, parts, kb0, kb1;
};

// Units of a launch of `tiles` tiles whose last `tail` tiles are split into
// `split` parts. Unit u < tiles - tail is tile u; then come the parts, tile
// by tile.
__device__ __forceinline__ int sk_units(int tiles, int tail, int split) { return tiles + tail * (split - 1); }

__device__ __forceinline__ SkUnit sk_unit_of(int tiles, int tail, int split, int u, int num_kb) {
  const int full = tiles - tail;
  if (u < full) return {u, 0, 1, 0, num_kb};
  const int v = u - full, i = v / split, s = v - i * split;
  return {full + i, s, split, s * num_kb / split, (s + 1) * num_kb / split};
}

__device__ __forceinline__ int sk_num_units(const TcParams& p) {
  return sk_units(p.tiles_m * p.tiles_n, p.sk_tail, p.sk_split);
}

__device__ __forceinline__ SkUnit sk_unit(const TcParams& p, int u, int num_kb) {
  return sk_unit_of(p.tiles_m * p.tiles_n, p.sk_tail, p.sk_split, u, num_kb);
}

// Counts one arrival of `parts` on an epoch-tagged counter (epoch in the high
// 24 bits, arrivals in the low 8). A counter holding another epoch (zero, or a
// launch that stopped early) counts as empty. The last arrival resets it to
// zero. Returns true for the last arrival. Called by one lane.
__device__ __forceinline__ bool sk_arrive_last(uint32_t* ctr, uint32_t epoch, int parts) {
  const uint32_t tag = epoch << 8;
  uint32_t cur = *reinterpret_cast<volatile uint32_t*>(ctr), seen, next;
  do {
    seen = cur;
    next = ((seen & 0xFFFFFF00u) == tag ? seen : tag) + 1u;
    cur = atomicCAS(ctr, seen, next);
  } while (cur != seen);
  const bool last = static_cast<int>(next & 0xFFu) == parts;
  if (last) atomicExch(ctr, 0u);
  return last;
}

// Stream-K part of one epilogue warp (32 accumulator rows of `ncols` f32
// columns at TMEM address `t_row`): publishes this part's rows at `mine`,
// counts the arrival, and returns true if this warp arrived last for its
// slab; it then holds the sum of all parts (`fix` = the row in part 0, parts
// `part_stride` floats apart, added in part order so the result does not
// depend on which part finished last) in TMEM in place of its own part, and
// the ordinary epilogue can run.
__device__ __noinline__ bool sk_publish_and_fix(uint32_t t_row, int ncols, float* mine, const float* fix,
                                                long long part_stride, int parts, uint32_t* counter, uint32_t epoch) {
#pragma unroll 1
  for (int c = 0; c < ncols; c += 32) {
    uint32_t r[32];
    tmem_ld_32x32b_x32(t_row + c, r);
    tmem_ld_wait();
    float4* dst = reinterpret_cast<float4*>(mine + c);
#pragma unroll
    for (int g = 0; g < 8; ++g)
      __stcg(dst + g, make_float4(__uint_as_float(r[4 * g]), __uint_as_float(r[4 * g + 1]),
                                  __uint_as_float(r[4 * g + 2]), __uint_as_float(r[4 * g + 3])));
  }
  __threadfence();
  __syncwarp();
  int last = 0;
  if ((threadIdx.x & 31) == 0) last = sk_arrive_last(counter, epoch, parts);
  last = __shfl_sync(0xffffffffu, last, 0);
  if (!last) return false;
  __threadfence();
#pragma unroll 1
  for (int c = 0; c < ncols; c += 32) {
    float acc[32];
#pragma unroll 1
    for (int s = 0; s < parts; ++s) {
      const float4* f = reinterpret_cast<const float4*>(fix + s * part_stride + c);
#pragma unroll
      for (int g = 0; g < 8; ++g) {
        const float4 v = __ldcg(f + g);
        acc[4 * g + 0] = s ? acc[4 * g + 0] + v.x : v.x;
        acc[4 * g + 1] = s ? acc[4 * g + 1] + v.y : v.y;
        acc[4 * g + 2] = s ? acc[4 * g + 2] + v.z : v.z;
        acc[4 * g + 3] = s ? acc[4 * g + 3] + v.w : v.w;
      }
    }
    uint32_t r[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(acc[i]);
    tmem_st_32x32b_x32(t_row + c, r);
  }
  tmem_st_wait();
  return true;
}

// Shared-memory staging per epilogue warp for kEpiScatterRows: a 32 x 32 f32
// block with a 33-float row pitch (bank-conflict-free both ways).
constexpr int kScatterStageFloats = 32 * 33;

constexpr int kFlagHFromRounded = 1;  // h computed from the bf16-rounded preact
constexpr int kFlagTmaEpilogue = 2;   // dswiglu: tmC / tmD are set and H % 32 == 0 (2-SM kernel)

template <int BN_, bool A_MN_, bool B_MN_, int EPI_, bool OUT_F32_>
struct TcCfg {
  static constexpr int BM = 128;
  static constexpr int BN = BN_;
  static constexpr int BK = 64;  // 64 bf16 = one 128-byte swizzle row
  static constexpr bool A_MN = A_MN_;
  static constexpr bool B_MN = B_MN_;
  static constexpr int EPI = EPI_;
  static constexpr bool OUT_F32 = OUT_F32_;
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int TX_BYTES = STAGE_BYTES;
  static constexpr int SMEM_BUDGET = 200 * 1024;
  static constexpr int STAGES = (SMEM_BUDGET / STAGE_BYTES) > 8 ? 8 : (SMEM_BUDGET / STAGE_BYTES);
  static constexpr int TMEM_COLS = 2 * BN;  // double-buffered accumulator
  static constexpr int NUM_EPI_WARPS = 4;
  static constexpr int NUM_THREADS = 32 * (2 + NUM_EPI_WARPS);
  static constexpr int BAR_BYTES = 8 * (2 * STAGES + 5) + 16;
  static constexpr int EPI_STAGE_BYTES = EPI == kEpiScatterRows ? NUM_EPI_WARPS * kScatterStageFloats * 4 : 0;
  static constexpr int SMEM_BYTES = 1024 + STAGES * STAGE_BYTES + BAR_BYTES + EPI_STAGE_BYTES;
  static_assert(STAGES >= 2, "pipeline needs at least two stages");
  static_assert(BN == 128 || BN == 256, "BN must be 128 or 256");
  static_assert(TMEM_COLS <= 512, "TMEM holds 512 columns");
};

__device__ __forceinline__ void tile_coords(int tile, int tiles_m, int tiles_n, int group_m, int& pm, int& pn) {
  // Grouped ordering of output tiles for L2 reuse (fused_forward.py:82-94).
  const int in_group = group_m * tiles_n;
  const int gid = tile / in_group;
  const int first_m = gid * group_m;
  const int gsz = min(tiles_m - first_m, group_m);
  const int r = tile % in_group;
  pm = first_m + r % gsz;
  pn = r / gsz;
}

// Store 32 consecutive output columns of one row (cols [c0, c0+32) of a row
// that starts at `row_ptr`), masking columns >= ncols in groups of 8.
template <bool F32>
__device__ __forceinline__ void store_row32(void* row_ptr, int c0, int ncols, const float (&v)[32]) {
  if constexpr (F32) {
    float* p = reinterpret_cast<float*>(row_ptr) + c0;
#pragma unroll
    for (int g = 0; g < 8; ++g) {
      if (c0 + 4 * g + 4 <= ncols) {
        *reinterpret_cast<float4*>(p + 4 * g) = make_float4(v[4 * g], v[4 * g + 1], v[4 * g + 2], v[4 * g + 3]);
      }
    }
  } else {
    __nv_bfloat16* p = reinterpret_cast<__nv_bfloat16*>(row_ptr) + c0;
#pragma unroll
    for (int g = 0; g < 4; ++g) {
      if (c0 + 8 * g + 8 <= ncols) {
        uint4 u;
        u.x = pack_bf16x2(v[8 * g + 0], v[8 * g + 1]);
        u.y = pack_bf16x2(v[8 * g + 2], v[8 * g + 3]);
        u.z = pack_bf16x2(v[8 * g + 4], v[8 * g + 5]);
        u.w = pack_bf16x2(v[8 * g + 6], v[8 * g + 7]);
        *reinterpret_cast<uint4*>(p + 8 * g) = u;
      }
    }
  }
}

// Epilogue of one output tile for the 32 rows of one warp: row `row` of the
// output (this thread's TMEM lane) and its TMEM address `t_row` (lane base +
// accumulator column base). Tile (pm, pn) of BN accumulator columns.
// Store epilogue through shared memory and TMA (2-SM kernel): each warp
// turns 32 accumulator columns of its 32 rows into a {32 x 32} box in one of
// two swizzled shared-memory buffers and one lane issues a TMA store of the
// box, so the output leaves as whole lines instead of 16 bytes of 32 rows per
// store instruction. Box rows are 64 bytes (bf16, 64-byte swizzle: 16-byte
// chunk c of row r at c ^ ((r >> 1) & 3)) or 128 bytes (f32, 128-byte
// swizzle: chunk c at c ^ (r & 7)); either way a warp's 16-byte writes take
// the minimum four wavefronts. `stage` is 1024-byte aligned, two boxes.
template <bool OUT_F32>
struct StoreStage {
  static constexpr int kRowBytes = OUT_F32 ? 128 : 64;
  static constexpr int kBoxBytes = 32 * kRowBytes;
  static constexpr int kWarpBytes = 2 * ((kBoxBytes + 1023) / 1024) * 1024;
};

// SCALED (e4m3 operands): D[row, col] is scaled by scale_a[row] * scale_b[col]
// before it is stored.
template <int BN, bool OUT_F32, bool SCALED = false>
__device__ __forceinline__ void epilogue_store_tma(const TcParams& p, int pn, int row0, uint32_t t_row,
                                                   uint8_t* stage) {
  using S = StoreStage<OUT_F32>;
  constexpr int kChunks16 = S::kRowBytes / 16;  // 16-byte chunks per box row
  const uint32_t lane = threadIdx.x & 31u;
  const int n0 = pn * BN;
  float sa = 1.0f;
  if constexpr (SCALED) sa = row0 + static_cast<int>(lane) < p.M ? p.scale_a[row0 + lane] : 0.0f;
#pragma unroll 1
  for (int c = 0; c < BN / 32; ++c) {
    uint32_t r[32];
    tmem_ld_32x32b_x32(t_row + c * 32, r);
    tmem_ld_wait();
    if constexpr (SCALED) {
      const int col = n0 + c * 32 + static_cast<int>(lane);
      const float sb = col < p.N ? p.scale_b[col] : 0.0f;
#pragma unroll
      for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * sa * __shfl_sync(0xffffffffu, sb, i));
    }
    uint8_t* buf = stage + (c & 1) * (S::kWarpBytes / 2);
    // The store issued from this buffer two chunks ago (possibly in the
    // previous tile) has read it once at most one store is still reading.
    if (lane == 0) bulk_wait_read<1>();
    __syncwarp();
    uint8_t* row_base = buf + lane * S::kRowBytes;
#pragma unroll
    for (int k = 0; k < kChunks16; ++k) {
      uint4 v;
      if constexpr (OUT_F32) {
        v = make_uint4(r[4 * k], r[4 * k + 1], r[4 * k + 2], r[4 * k + 3]);
      } else {
        v = make_uint4(pack_bf16x2(__uint_as_float(r[8 * k]), __uint_as_float(r[8 * k + 1])),
                       pack_bf16x2(__uint_as_float(r[8 * k + 2]), __uint_as_float(r[8 * k + 3])),
                       pack_bf16x2(__uint_as_float(r[8 * k + 4]), __uint_as_float(r[8 * k + 5])),
                       pack_bf16x2(__uint_as_float(r[8 * k + 6]), __uint_as_float(r[8 * k + 7])));
      }
      const int kk = OUT_F32 ? (k ^ static_cast<int>(lane & 7u)) : (k ^ static_cast<int>((lane >> 1) & 3u));
      *reinterpret_cast<uint4*>(row_base + 16 * kk) = v;
    }
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
      tma_store_2d(&p.tmC, buf, n0 + c * 32, row0);
      bulk_commit();
    }
  }
}

// SwiGLU epilogue through shared memory and TMA (2-SM kernel; H % 32 == 0
// so every 32-unit chunk below H is whole): per chunk of 32 hidden units a
// warp fills up to three {32 x 32} bf16 boxes (preact left, preact gate, h;
// 64-byte rows, 64-byte swizzle as in epilogue_store_tma) and one lane issues
// their TMA stores. The single 6 KB staging area is reused once the previous
// chunk's stores have read it. Chunks at or beyond H are skipped (in the
// standard layout their left columns would fall on gate columns).
struct SwigluStage {
  static constexpr int kBoxBytes = 32 * 64;
  static constexpr int kWarpBytes = 3 * kBoxBytes;
};

__device__ __forceinline__ void stage_row32_bf16(uint8_t* box, uint32_t lane, const float (&v)[32]) {
  uint8_t* row = box + lane * 64;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const uint4 u = make_uint4(pack_bf16x2(v[8 * k], v[8 * k + 1]), pack_bf16x2(v[8 * k + 2], v[8 * k + 3]),
                               pack_bf16x2(v[8 * k + 4], v[8 * k + 5]), pack_bf16x2(v[8 * k + 6], v[8 * k + 7]));
    *reinterpret_cast<uint4*>(row + 16 * (k ^ static_cast<int>((lane >> 1) & 3u))) = u;
  }
}

// SCALED (e4m3 operands): the left and gate accumulators of row `row` and
// unit j are scaled by scale_a[row] * scale_b[B row of left / gate j] first.
template <int BN, bool SCALED = false>
__device__ __forceinline__ void epilogue_swiglu_tma(const TcParams& p, int pn, int row0, uint32_t t_row,
                                                    uint8_t* stage) {
  const uint32_t lane = threadIdx.x & 31u;
  const int j0 = pn * (BN / 2);
  const bool rounded = (p.flags & kFlagHFromRounded) != 0;
  uint8_t* lbox = stage;
  uint8_t* gbox = stage + SwigluStage::kBoxBytes;
  uint8_t* hbox = stage + 2 * SwigluStage::kBoxBytes;
  float sa = 1.0f;
  if constexpr (SCALED) sa = row0 + static_cast<int>(lane) < p.M ? p.scale_a[row0 + lane] : 0.0f;
#pragma unroll 1
  for (int c = 0; c < BN / 64; ++c) {
    const int j = j0 + c * 32;
    if (j >= p.H) break;
    uint32_t rl[32], rg[32];
    tmem_ld_32x32b_x32(t_row + c * 32, rl);
    tmem_ld_32x32b_x32(t_row + BN / 2 + c * 32, rg);
    tmem_ld_wait();
    float sbl = 1.0f, sbg = 1.0f;
    if constexpr (SCALED) {
      const int jj = j + static_cast<int>(lane);
      sbl = jj < p.H ? p.scale_b[left_col(jj, p.H, p.layout)] : 0.0f;
      sbg = jj < p.H ? p.scale_b[gate_col(jj, p.H, p.layout)] : 0.0f;
    }
    float lf[32], gf[32], hf[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      float l = __uint_as_float(rl[i]);
      float g = __uint_as_float(rg[i]);
      if constexpr (SCALED) {
        l = l * sa * __shfl_sync(0xffffffffu, sbl, i);
        g = g * sa * __shfl_sync(0xffffffffu, sbg, i);
      }
      lf[i] = l;
      gf[i] = g;
      if (rounded) {
        l = bf16_round(l);
        g = bf16_round(g);
      }
      hf[i] = l * (g * sigmoid_fast(g));
    }
    if (lane == 0) bulk_wait_read<0>();  // the previous chunk's stores have read the boxes
    __syncwarp();
    if (p.out0) {
      stage_row32_bf16(lbox, lane, lf);
      stage_row32_bf16(gbox, lane, gf);
    }
    if (p.out1) stage_row32_bf16(hbox, lane, hf);
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
      if (p.out0) {
        tma_store_2d(&p.tmC, lbox, left_col(j, p.H, p.layout), row0);
        tma_store_2d(&p.tmC, gbox, gate_col(j, p.H, p.layout), row0);
      }
      if (p.out1) tma_store_2d(&p.tmD, hbox, j, row0);
      bulk_commit();
    }
  }
}

// dSwiGLU epilogue of the 2-SM kernel (needs H % 32 == 0), all through TMA:
// per chunk of 32 hidden units a warp TMA-loads the preact left and gate
// {32 x 32} boxes of its 32 rows into one of two buffers (the next chunk's
// load is in flight while this one is computed), each thread reads its row,
// writes grad_left / grad_gate back into the same boxes and h into a third,
// and one lane TMA-stores the three (grad_preact over preact, in place). No
// per-lane global loads or stores remain. Box rows are 64 bytes with the
// 64-byte swizzle of epilogue_store_tma. `lbar` holds this warp's two
// load barriers; `lphase` their parities, kept across tiles.
struct DswigluStage {
  static constexpr int kBoxBytes = 32 * 64;
  static constexpr int kBufBytes = 3 * kBoxBytes;  // left, gate, h
  static constexpr int kWarpBytes = 2 * kBufBytes;
};

template <int BN>
__device__ __forceinline__ bool epilogue_dswiglu_tma(const TcParams& p, int pn, int row0, uint32_t t_row,
                                                     uint8_t* stage, uint64_t* lbar, uint32_t& lphase,
                                                     volatile int* abort_flag) {
  const uint32_t lane = threadIdx.x & 31u;
  const int j0 = pn * BN;
  int nch = 0;  // whole chunks below N
  while (nch < BN / 32 && j0 + 32 * nch < p.N) ++nch;
  const int swz = static_cast<int>((lane >> 1) & 3u);
  auto issue_load = [&](int c) {  // lane 0; the buffer's earlier stores must have read it
    uint8_t* buf = stage + (c & 1) * DswigluStage::kBufBytes;
    const int j = j0 + 32 * c;
    bulk_wait_read<0>();
    mbar_arrive_expect_tx(&lbar[c & 1], 2 * DswigluStage::kBoxBytes);
    tma_load_2d(buf, &p.tmC, &lbar[c & 1], left_col(j, p.H, p.layout), row0);
    tma_load_2d(buf + DswigluStage::kBoxBytes, &p.tmC, &lbar[c & 1], gate_col(j, p.H, p.layout), row0);
  };
  if (nch > 0 && lane == 0) issue_load(0);
#pragma unroll 1
  for (int c = 0; c < nch; ++c) {
    const int j = j0 + 32 * c;
    if (c + 1 < nch && lane == 0) issue_load(c + 1);
    uint32_t r[32];
    tmem_ld_32x32b_x32(t_row + c * 32, r);
    tmem_ld_wait();
    const uint32_t b = static_cast<uint32_t>(c & 1);
    if (!mbar_wait(&lbar[b], (lphase >> b) & 1u, abort_flag, p.status, kErrTimeoutEpilogue)) return false;
    lphase ^= 1u << b;
    uint8_t* lbox = stage + b * DswigluStage::kBufBytes;
    uint8_t* gbox = lbox + DswigluStage::kBoxBytes;
    uint8_t* hbox = gbox + DswigluStage::kBoxBytes;
#pragma unroll
    for (int v8 = 0; v8 < 4; ++v8) {
      const int off = static_cast<int>(lane) * 64 + 16 * (v8 ^ swz);
      const uint4 lu = *reinterpret_cast<const uint4*>(lbox + off);
      const uint4 gu = *reinterpret_cast<const uint4*>(gbox + off);
      const uint32_t lw[4] = {lu.x, lu.y, lu.z, lu.w};
      const uint32_t gw[4] = {gu.x, gu.y, gu.z, gu.w};
      uint32_t glw[4], ggw[4], hw[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 l2 = unpack_bf16x2(lw[e]);
        const float2 g2 = unpack_bf16x2(gw[e]);
        const float ls[2] = {l2.x, l2.y};
        const float gs[2] = {g2.x, g2.y};
        float glv[2], ggv[2], hv[2];
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          const int i = 8 * v8 + 2 * e + u;
          // grad_h is a bf16 tensor in the reference before the pointwise step.
          const float dh = bf16_round(__uint_as_float(r[i]));
          const float sg = sigmoid_fast(gs[u]);
          const float silu = gs[u] * sg;
          const float dsilu = sg + silu * (1.0f - sg);
          glv[u] = dh * silu;
          ggv[u] = dh * ls[u] * dsilu;
          hv[u] = ls[u] * silu;  // h for the plain dW2 GEMM ("emit_h" mode)
        }
        glw[e] = pack_bf16x2(glv[0], glv[1]);
        ggw[e] = pack_bf16x2(ggv[0], ggv[1]);
        hw[e] = pack_bf16x2(hv[0], hv[1]);
      }
      *reinterpret_cast<uint4*>(lbox + off) = make_uint4(glw[0], glw[1], glw[2], glw[3]);
      *reinterpret_cast<uint4*>(gbox + off) = make_uint4(ggw[0], ggw[1], ggw[2], ggw[3]);
      if (p.out1) *reinterpret_cast<uint4*>(hbox + off) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
    }
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
      tma_store_2d(&p.tmC, lbox, left_col(j, p.H, p.layout), row0);
      tma_store_2d(&p.tmC, gbox, gate_col(j, p.H, p.layout), row0);
      if (p.out1) tma_store_2d(&p.tmD, hbox, j, row0);
      bulk_commit();
    }
  }
  return true;
}

template <int BN, int EPI, bool OUT_F32>
__device__ __forceinline__ void epilogue_tile(const TcParams& p, int pm, int pn, int row, uint32_t t_row,
                                              float* stage = nullptr) {
  const bool row_ok = row < p.M;
  if constexpr (EPI == kEpiStore) {
    const int n0 = pn * BN;
    char* out_row = reinterpret_cast<char*>(p.out0) +
                    (static_cast<long long>(row) * p.ld0) * (OUT_F32 ? 4 : 2);
#pragma unroll 1
    for (int c = 0; c < BN / 32; ++c) {
      uint32_t r[32];
      tmem_ld_32x32b_x32(t_row + c * 32, r);
      tmem_ld_wait();
      float v[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
      if (row_ok) store_row32<OUT_F32>(out_row, n0 + c * 32, p.N, v);
    }
  } else if constexpr (EPI == kEpiSwiglu) {
    const int j0 = pn * (BN / 2);
    __nv_bfloat16* pre_row = reinterpret_cast<__nv_bfloat16*>(p.out0) + static_cast<long long>(row) * p.ld0;
    __nv_bfloat16* h_row =
        p.out1 ? reinterpret_cast<__nv_bfloat16*>(p.out1) + static_cast<long long>(row) * p.ld1 : nullptr;
    const bool rounded = (p.flags & kFlagHFromRounded) != 0;
#pragma unroll 1
    for (int c = 0; c < BN / 64; ++c) {
      uint32_t rl[32], rg[32];
      tmem_ld_32x32b_x32(t_row + c * 32, rl);
      tmem_ld_32x32b_x32(t_row + BN / 2 + c * 32, rg);
      tmem_ld_wait();
      const int j = j0 + c * 32;  // first hidden unit of this chunk (multiple of 32)
      float lf[32], gf[32], hf[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        float l = __uint_as_float(rl[i]);
        float g = __uint_as_float(rg[i]);
        lf[i] = l;
        gf[i] = g;
        if (rounded) {
          l = bf16_round(l);
          g = bf16_round(g);
        }
        hf[i] = l * (g * sigmoid_fast(g));
      }
      if (row_ok) {
        if (p.out0) {  // preact is not stored by the no-save (inference) forward
          store_row32<false>(pre_row, left_col(j, p.H, p.layout), left_col(j, p.H, p.layout) + (p.N - j), lf);
          store_row32<false>(pre_row, gate_col(j, p.H, p.layout), gate_col(j, p.H, p.layout) + (p.N - j), gf);
        }
        if (h_row) store_row32<false>(h_row, j, p.N, hf);
      }
    }
  } else if constexpr (EPI == kEpiScatterRows) {
    // Tensor-parallel reduce-scatter fused into the GEMM: each f32 partial
    // row goes straight into its owning rank's receive slot, usually another
    // GPU's memory. Each 32 x 32 block is transposed through shared memory so
    // that a warp store writes four whole 128-byte row segments (lane l: row
    // 4i + l/8, columns 4(l%8)..+3) instead of 16 bytes of 32 different rows.
    const int lane = static_cast<int>(threadIdx.x & 31);
    const int row0 = row - lane;  // first row of this warp's 32-row group
    const int n0 = pn * BN;
#pragma unroll 1
    for (int c = 0; c < BN / 32; ++c) {
      uint32_t r[32];
      tmem_ld_32x32b_x32(t_row + c * 32, r);
      tmem_ld_wait();
#pragma unroll
      for (int i = 0; i < 32; ++i) stage[lane * 33 + i] = __uint_as_float(r[i]);
      __syncwarp();
      const int col = n0 + c * 32 + 4 * (lane & 7);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int rr = 4 * i + (lane >> 3);
        const int grow = row0 + rr;
        if (grow < p.M && col + 4 <= p.N) {
          const int owner = grow / p.rows_per_rank;
          const long long dst_row =
              static_cast<long long>(p.src_rank) * p.rows_per_rank + (grow - owner * p.rows_per_rank);
          const float* src = stage + rr * 33 + 4 * (lane & 7);
          *reinterpret_cast<float4*>(p.peer[owner] + dst_row * p.ld0 + col) =
              make_float4(src[0], src[1], src[2], src[3]);
        }
      }
      __syncwarp();
    }
  } else {  // kEpiDswiglu
    // grad_h never leaves registers: each 32-column chunk of it is combined
    // with the matching preact left/gate values and written back over them.
    // The preact loads of chunk c+1 are issued before chunk c is computed so
    // their latency hides behind the TMEM load and the SiLU math.
    const int j0 = pn * BN;
    __nv_bfloat16* pre_row = reinterpret_cast<__nv_bfloat16*>(p.out0) + static_cast<long long>(row) * p.ld0;
    __nv_bfloat16* h_row =
        p.out1 ? reinterpret_cast<__nv_bfloat16*>(p.out1) + static_cast<long long>(row) * p.ld1 : nullptr;
    uint4 lu[2][4], gu[2][4];
    auto load_chunk = [&](int c, int buf) {
      const int j = j0 + c * 32;
      const int lc = left_col(j, p.H, p.layout);
      const int gc = gate_col(j, p.H, p.layout);
#pragma unroll
      for (int v8 = 0; v8 < 4; ++v8) {
        if (row_ok && j + 8 * v8 + 8 <= p.N) {
          lu[buf][v8] = *reinterpret_cast<const uint4*>(pre_row + lc + 8 * v8);
          gu[buf][v8] = *reinterpret_cast<const uint4*>(pre_row + gc + 8 * v8);
        }
      }
    };
    load_chunk(0, 0);
#pragma unroll
    for (int c = 0; c < BN / 32; ++c) {
      const int buf = c & 1;
      if (c + 1 < BN / 32) load_chunk(c + 1, buf ^ 1);
      uint32_t r[32];
      tmem_ld_32x32b_x32(t_row + c * 32, r);
      tmem_ld_wait();
      const int j = j0 + c * 32;
      if (row_ok) {
        const int lc = left_col(j, p.H, p.layout);
        const int gc = gate_col(j, p.H, p.layout);
        // Each group of 8 columns is stored as soon as it is formed (16-byte
        // stores of grad_left, grad_gate and h), masking columns >= N.
#pragma unroll
        for (int v8 = 0; v8 < 4; ++v8) {
          const uint32_t lw[4] = {lu[buf][v8].x, lu[buf][v8].y, lu[buf][v8].z, lu[buf][v8].w};
          const uint32_t gw[4] = {gu[buf][v8].x, gu[buf][v8].y, gu[buf][v8].z, gu[buf][v8].w};
          uint32_t glw[4], ggw[4], hw[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 l2 = unpack_bf16x2(lw[e]);
            const float2 g2 = unpack_bf16x2(gw[e]);
            const float ls[2] = {l2.x, l2.y};
            const float gs[2] = {g2.x, g2.y};
            float glv[2], ggv[2], hv[2];
#pragma unroll
            for (int u = 0; u < 2; ++u) {
              const int i = 8 * v8 + 2 * e + u;
              // grad_h is a bf16 tensor in the reference before the pointwise step.
              const float dh = bf16_round(__uint_as_float(r[i]));
              const float sg = sigmoid_fast(gs[u]);
              const float silu = gs[u] * sg;
              const float dsilu = sg + silu * (1.0f - sg);
              glv[u] = dh * silu;
              ggv[u] = dh * ls[u] * dsilu;
              hv[u] = ls[u] * silu;  // h for the plain dW2 GEMM ("emit_h" mode)
            }
            glw[e] = pack_bf16x2(glv[0], glv[1]);
            ggw[e] = pack_bf16x2(ggv[0], ggv[1]);
            hw[e] = pack_bf16x2(hv[0], hv[1]);
          }
          if (j + 8 * v8 + 8 <= p.N) {
            *reinterpret_cast<uint4*>(pre_row + lc + 8 * v8) = make_uint4(glw[0], glw[1], glw[2], glw[3]);
            *reinterpret_cast<uint4*>(pre_row + gc + 8 * v8) = make_uint4(ggw[0], ggw[1], ggw[2], ggw[3]);
            if (h_row) *reinterpret_cast<uint4*>(h_row + j + 8 * v8) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
          }
        }
      }
    }
  }
}

template <class Cfg>
__global__ void __launch_bounds__(Cfg::NUM_THREADS, 1) tc_gemm_kernel(const __grid_constant__ TcParams p) {
  constexpr int BM = Cfg::BM, BN = Cfg::BN, BK = Cfg::BK, STAGES = Cfg::STAGES;

  extern __shared__ uint8_t smem_raw[];
  // 128-byte swizzled TMA boxes and UMMA atoms need 1024-byte alignment.
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + STAGES * Cfg::STAGE_BYTES);
  uint64_t* full = bars;                    // TMA -> MMA
  uint64_t* empty = bars + STAGES;          // MMA -> TMA
  uint64_t* tmem_full = bars + 2 * STAGES;  // MMA -> epilogue (2)
  uint64_t* tmem_empty = tmem_full + 2;     // epilogue -> MMA (2)
  uint64_t* mma_done = tmem_empty + 2;      // MMA teardown
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const uint32_t warp = warp_id();
  const uint32_t lane = lane_id();

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tmem_full[a], 1);
      mbar_init(&tmem_empty[a], Cfg::NUM_EPI_WARPS);
    }
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, Cfg::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before_sync();
  __syncthreads();
  tc_fence_after_sync();
  const uint32_t tmem_base = *tmem_slot;

  const int num_tiles = p.tiles_m * p.tiles_n;
  const int num_kb = (p.K + BK - 1) / BK;
  uint32_t* status = p.status;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      tma_prefetch_desc(&p.tmA);
      tma_prefetch_desc(&p.tmB);
      uint32_t stage = 0, phase = 0;
      uint32_t filled = 0, fill_parity = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        int pm, pn;
        tile_coords(tile, p.tiles_m, p.tiles_n, p.group_m, pm, pn);
        const int m0 = pm * BM;
        // Origins of the two B halves (BN/2 columns each).
        int b0, b1;
        if constexpr (Cfg::EPI == kEpiSwiglu) {
          const int j0 = pn * (BN / 2);
          b0 = left_col(j0, p.H, p.layout);
          b1 = gate_col(j0, p.H, p.layout);
        } else {
          b0 = pn * BN;
          b1 = b0 + BN / 2;
        }
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag, status, kErrTimeoutProducer)) {
            ok = false;
            break;
          }
          uint8_t* sa = smem + stage * Cfg::STAGE_BYTES;
          uint8_t* sb = sa + Cfg::A_BYTES;
          mbar_arrive_expect_tx(&full[stage], Cfg::TX_BYTES);
          const int k0 = kb * BK;
          if constexpr (Cfg::A_MN) {
            tma_load_2d(sa, &p.tmA, &full[stage], m0, k0);
            tma_load_2d(sa + 64 * BK * 2, &p.tmA, &full[stage], m0 + 64, k0);
          } else {
            tma_load_2d(sa, &p.tmA, &full[stage], k0, m0);
          }
          if constexpr (Cfg::B_MN) {
#pragma unroll
            for (int i = 0; i < BN / 128; ++i) {
              tma_load_2d(sb + i * 8192, &p.tmB, &full[stage], b0 + 64 * i, k0);
            }
#pragma unroll
            for (int i = 0; i < BN / 128; ++i) {
              tma_load_2d(sb + (BN / 128 + i) * 8192, &p.tmB, &full[stage], b1 + 64 * i, k0);
            }
          } else {
            tma_load_2d(sb, &p.tmB, &full[stage], k0, b0);
            tma_load_2d(sb + (BN / 2) * 128, &p.tmB, &full[stage], k0, b1);
          }
          filled |= 1u << stage;
          fill_parity = (fill_parity & ~(1u << stage)) | (phase << stage);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      // Drain: every load this thread issued must land before the CTA exits.
      for (int s = 0; s < STAGES; ++s) {
        if (filled & (1u << s)) {
          volatile int never = 0;
          mbar_wait(&full[s], (fill_parity >> s) & 1u, &never, status, kErrTimeoutTeardown);
        }
      }
    }
  } else if (warp == 1) {
    // ----------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc_f16(BM, BN, 1, 1, Cfg::A_MN ? 1 : 0, Cfg::B_MN ? 1 : 0);
      uint32_t stage = 0, phase = 0, acc = 0, acc_phase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        if (!mbar_wait(&tmem_empty[acc], acc_phase ^ 1, abort_flag, status, kErrTimeoutMma)) break;
        tc_fence_after_sync();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort_flag, status, kErrTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after_sync();
          const uint32_t sa = smem_u32(smem + stage * Cfg::STAGE_BYTES);
          const uint32_t sb = sa + Cfg::A_BYTES;
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            // K-major: advance 16 elements = 32 bytes inside the swizzle row.
            // MN-major: advance 16 rows of 128 bytes.
            const uint64_t adesc = Cfg::A_MN ? make_smem_desc_sw128(sa + k * 2048, p.mn_lbo, p.mn_sbo)
                                             : make_smem_desc_sw128(sa + k * 32, 16, 1024);
            const uint64_t bdesc = Cfg::B_MN ? make_smem_desc_sw128(sb + k * 2048, p.mn_lbo, p.mn_sbo)
                                             : make_smem_desc_sw128(sb + k * 32, 16, 1024);
            umma_f16_ss(d_tmem, adesc, bdesc, idesc, (kb | k) != 0 ? 1u : 0u);
          }
          umma_commit(&empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        umma_commit(&tmem_full[acc]);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1;
        }
      }
      // All MMAs issued by this thread complete before TMEM is released.
      umma_commit(mma_done);
      volatile int never = 0;
      mbar_wait(mma_done, 0, &never, status, kErrTimeoutTeardown);
    }
  } else if (warp < 2 + Cfg::NUM_EPI_WARPS) {
    // ------------------------------------------------------------- epilogue
    const uint32_t q = warp & 3u;  // TMEM lane quarter this warp may access
    uint32_t acc = 0, acc_phase = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
      int pm, pn;
      tile_coords(tile, p.tiles_m, p.tiles_n, p.group_m, pm, pn);
      if (!mbar_wait(&tmem_full[acc], acc_phase, abort_flag, status, kErrTimeoutEpilogue)) break;
      tc_fence_after_sync();
      const int row = pm * BM + static_cast<int>(q * 32 + lane);
      const uint32_t t_row = tmem_base + ((q * 32u) << 16) + acc * BN;
      float* stage = reinterpret_cast<float*>(smem + STAGES * Cfg::STAGE_BYTES + Cfg::BAR_BYTES) +
                     (warp - 2) * kScatterStageFloats;
      epilogue_tile<BN, Cfg::EPI, Cfg::OUT_F32>(p, pm, pn, row, t_row, stage);
      tc_fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tmem_empty[acc]);
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1;
      }
    }
  }

  tc_fence_before_sync();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after_sync();
    tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
  }
}

}  // namespace swiglu
