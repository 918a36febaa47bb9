// fp32-input path and the standalone pointwise kernels.
//
// The fp32 mode reproduces the reference's "ieee" fp32 path
// (fused_forward.py:229-233, input_precision="ieee"): tcgen05 has no true-fp32
// MMA kind, so these GEMMs run on the FFMA pipe with a 64x64 register-blocked
// tile. They exist for the 1e-5 correctness mode, not for throughput.
//
// The pointwise kernels are HBM-bound: 16-byte vector loads/stores, one
// grid-stride loop, fp32 internal math and a single rounding on store, which is
// how Inductor evaluates the reference's compiled helpers
// (swiglu_recompute.py:26-49).
#pragma once

#include "tc_gemm.cuh"

namespace swiglu {

struct SimtParams {
  const float* a;
  const float* b;  // B operand, or preact when TRANSFORM
  float* out0;
  float* out1;
  long long lda, ldb, ld0, ld1;
  int M, N, K, H, layout;
};

// C[M,N] = A[M,K] B[K,N]; A_MN: A stored [K][M]; B_MN: B stored [K][N].
// Thread (tx, ty) owns rows 4ty..4ty+3 and columns {2tx, 2tx+1, 32+2tx, 33+2tx}
// of the 64x64 tile, so the SwiGLU epilogue finds each left column and its
// gate column (tile columns c and c+32) in the same thread.
template <bool A_MN, bool B_MN, int EPI, bool TRANSFORM>
__global__ void __launch_bounds__(256) simt_gemm_f32_kernel(const SimtParams p) {
  constexpr int TM = 64, TN = 64, TK = 16;
  __shared__ float As[TK][TM + 4];
  __shared__ float Bs[TK][TN + 4];
  const int tid = threadIdx.x;
  const int tx = tid % 16, ty = tid / 16;
  const int m0 = blockIdx.y * TM;
  const int nt = blockIdx.x;
  // Source column of tile column c (EPI_SWIGLU: 32 hidden units per tile).
  auto bcol = [&](int c, int& src, bool& valid) {
    if constexpr (EPI == kEpiSwiglu) {
      const int j = nt * 32 + (c & 31);
      valid = j < p.N;
      src = c < 32 ? left_col(j, p.H, p.layout) : gate_col(j, p.H, p.layout);
    } else {
      const int j = nt * TN + c;
      valid = j < p.N;
      src = j;
    }
  };
  float acc[4][4] = {};
  for (int k0 = 0; k0 < p.K; k0 += TK) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int e = tid + 256 * i;
      int m, k;
      if (A_MN) { k = e / TM; m = e % TM; } else { m = e / TK; k = e % TK; }
      const int gm = m0 + m, gk = k0 + k;
      float v = 0.f;
      if (gm < p.M && gk < p.K) v = A_MN ? p.a[(long long)gk * p.lda + gm] : p.a[(long long)gm * p.lda + gk];
      As[k][m] = v;
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int e = tid + 256 * i;
      int n, k;
      if (B_MN) { k = e / TN; n = e % TN; } else { n = e / TK; k = e % TK; }
      const int gk = k0 + k;
      float v = 0.f;
      if constexpr (TRANSFORM) {
        const int j = nt * TN + n;
        if (j < p.N && gk < p.K) {
          const float l = p.b[(long long)gk * p.ldb + left_col(j, p.H, p.layout)];
          const float g = p.b[(long long)gk * p.ldb + gate_col(j, p.H, p.layout)];
          v = l * (g * (1.0f / (1.0f + expf(-g))));
        }
      } else {
        int src;
        bool valid;
        bcol(n, src, valid);
        if (valid && gk < p.K) v = B_MN ? p.b[(long long)gk * p.ldb + src] : p.b[(long long)src * p.ldb + gk];
      }
      Bs[k][n] = v;
    }
    __syncthreads();
#pragma unroll
    for (int k = 0; k < TK; ++k) {
      float av[4], bv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) av[i] = As[k][4 * ty + i];
      bv[0] = Bs[k][2 * tx];
      bv[1] = Bs[k][2 * tx + 1];
      bv[2] = Bs[k][32 + 2 * tx];
      bv[3] = Bs[k][33 + 2 * tx];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
    }
    __syncthreads();
  }
  const int cols[4] = {2 * tx, 2 * tx + 1, 32 + 2 * tx, 33 + 2 * tx};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int r = m0 + 4 * ty + i;
    if (r >= p.M) continue;
    if constexpr (EPI == kEpiStore) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int c = nt * TN + cols[j];
        if (c < p.N) p.out0[(long long)r * p.ld0 + c] = acc[i][j];
      }
    } else if constexpr (EPI == kEpiSwiglu) {
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int hj = nt * 32 + cols[j];
        if (hj >= p.N) continue;
        const float l = acc[i][j], g = acc[i][j + 2];
        if (p.out0) {
          p.out0[(long long)r * p.ld0 + left_col(hj, p.H, p.layout)] = l;
          p.out0[(long long)r * p.ld0 + gate_col(hj, p.H, p.layout)] = g;
        }
        if (p.out1) p.out1[(long long)r * p.ld1 + hj] = l * (g * (1.0f / (1.0f + expf(-g))));
      }
    } else {  // kEpiDswiglu: acc = grad_h, preact updated in place
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int hj = nt * TN + cols[j];
        if (hj >= p.N) continue;
        float* pl = p.out0 + (long long)r * p.ld0 + left_col(hj, p.H, p.layout);
        float* pg = p.out0 + (long long)r * p.ld0 + gate_col(hj, p.H, p.layout);
        const float l = *pl, g = *pg, dh = acc[i][j];
        const float sg = 1.0f / (1.0f + expf(-g));
        const float silu = g * sg;
        const float dsilu = sg + silu * (1.0f - sg);
        *pl = dh * silu;
        *pg = dh * l * dsilu;
      }
    }
  }
}

// ------------------------------------------------------------ pointwise
template <typename T> struct Vec8;
template <> struct Vec8<__nv_bfloat16> {
  static constexpr int N = 8;
  __device__ static void load(const __nv_bfloat16* p, float (&v)[8]) {
    const uint4 u = *reinterpret_cast<const uint4*>(p);
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = unpack_bf16x2(w[e]);
      v[2 * e] = f.x;
      v[2 * e + 1] = f.y;
    }
  }
  __device__ static void store(__nv_bfloat16* p, const float (&v)[8]) {
    uint4 u;
    u.x = pack_bf16x2(v[0], v[1]);
    u.y = pack_bf16x2(v[2], v[3]);
    u.z = pack_bf16x2(v[4], v[5]);
    u.w = pack_bf16x2(v[6], v[7]);
    *reinterpret_cast<uint4*>(p) = u;
  }
};
template <> struct Vec8<float> {
  static constexpr int N = 8;
  __device__ static void load(const float* p, float (&v)[8]) {
    const float4 a = reinterpret_cast<const float4*>(p)[0];
    const float4 b = reinterpret_cast<const float4*>(p)[1];
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  }
  __device__ static void store(float* p, const float (&v)[8]) {
    reinterpret_cast<float4*>(p)[0] = make_float4(v[0], v[1], v[2], v[3]);
    reinterpret_cast<float4*>(p)[1] = make_float4(v[4], v[5], v[6], v[7]);
  }
};

// h[M,H] = left * silu(gate) from preact[M,2H] (swiglu_recompute.py:26-30,
// fused_forward_packed.py:281-286). H % 8 == 0.
template <typename T>
__global__ void swiglu_fwd_pointwise_kernel(const T* __restrict__ preact, T* __restrict__ h, long long M, int H,
                                            int layout) {
  const long long groups_per_row = H / 8;
  const long long total = M * groups_per_row;
  for (long long g = blockIdx.x * (long long)blockDim.x + threadIdx.x; g < total;
       g += (long long)gridDim.x * blockDim.x) {
    const long long r = g / groups_per_row;
    const int j = static_cast<int>(g - r * groups_per_row) * 8;
    const T* row = preact + r * 2LL * H;
    float l[8], gt[8], o[8];
    Vec8<T>::load(row + left_col(j, H, layout), l);
    Vec8<T>::load(row + gate_col(j, H, layout), gt);
#pragma unroll
    for (int e = 0; e < 8; ++e) o[e] = l[e] * (gt[e] * (1.0f / (1.0f + expf(-gt[e]))));
    Vec8<T>::store(h + r * H + j, o);
  }
}

// grad_preact[M,2H] from preact[M,2H] and grad_h[M,H] with the explicit SiLU
// derivative (swiglu_recompute.py:33-49; packed: fused_forward_packed.py:222-259).
// grad_preact may alias preact.
template <typename T>
__global__ void swiglu_bwd_pointwise_kernel(const T* preact, const T* __restrict__ grad_h, T* grad_preact,
                                            long long M, int H, int layout) {
  const long long groups_per_row = H / 8;
  const long long total = M * groups_per_row;
  for (long long g = blockIdx.x * (long long)blockDim.x + threadIdx.x; g < total;
       g += (long long)gridDim.x * blockDim.x) {
    const long long r = g / groups_per_row;
    const int j = static_cast<int>(g - r * groups_per_row) * 8;
    const long long lc = r * 2LL * H + left_col(j, H, layout);
    const long long gc = r * 2LL * H + gate_col(j, H, layout);
    float l[8], gt[8], dh[8], ol[8], og[8];
    Vec8<T>::load(preact + lc, l);
    Vec8<T>::load(preact + gc, gt);
    Vec8<T>::load(grad_h + r * H + j, dh);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float sg = 1.0f / (1.0f + expf(-gt[e]));
      const float silu = gt[e] * sg;
      const float dsilu = sg + silu * (1.0f - sg);
      ol[e] = dh[e] * silu;
      og[e] = dh[e] * l[e] * dsilu;
    }
    Vec8<T>::store(grad_preact + lc, ol);
    Vec8<T>::store(grad_preact + gc, og);
  }
}

// Chunk-interleaved packing of a [K, 2N] weight (fused_forward_packed.py:77-107):
// pack:   out[k, c*2B + s*B + i] = w[k, s*N + c*B + i]     (s = 0 left, 1 gate)
// unpack: the inverse. Element-wise gather, any block size B dividing N.
template <typename T>
__global__ void pack_chunked_kernel(const T* __restrict__ src, T* __restrict__ dst, long long K, long long N,
                                    long long B, int unpack) {
  const long long total = K * 2 * N;
  for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < total;
       e += (long long)gridDim.x * blockDim.x) {
    const long long k = e / (2 * N);
    const long long col = e - k * 2 * N;  // standard-layout column
    const long long s = col / N, rem = col - s * N;
    const long long c = rem / B, i = rem - c * B;
    const long long pcol = c * 2 * B + s * B + i;
    if (unpack) dst[k * 2 * N + col] = src[k * 2 * N + pcol];
    else dst[k * 2 * N + pcol] = src[k * 2 * N + col];
  }
}

// ----------------------------------------------------- e4m3 quantisation
// Per-row e4m3 quantisation of a bf16 [rows, cols] matrix for the FP8 GEMMs
// (cols % 8 == 0), one warp per row: amax_r = max |v| over the row, the
// stored dequantisation factor s_r = amax_r / 448 (1 for an all-zero row) and
// q = e4m3(v * (448 / amax_r)) rounded to nearest even, saturating at the
// largest finite e4m3 value 448. Both divisions are IEEE f32, so a CPU
// restatement reproduces q and s_r bit for bit.
__global__ void quantize_rows_e4m3_kernel(const __nv_bfloat16* __restrict__ src, uint8_t* __restrict__ dst,
                                          float* __restrict__ row_scale, long long rows, int cols) {
  const int lane = static_cast<int>(threadIdx.x & 31);
  const long long nwarps = (static_cast<long long>(gridDim.x) * blockDim.x) >> 5;
  const int vecs = cols / 8;
  for (long long r = (blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x) >> 5; r < rows; r += nwarps) {
    const uint4* row = reinterpret_cast<const uint4*>(src + r * cols);
    float amax = 0.0f;
    for (int v = lane; v < vecs; v += 32) {
      const uint4 u = row[v];
      const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = unpack_bf16x2(w[e]);
        amax = fmaxf(amax, fmaxf(fabsf(f.x), fabsf(f.y)));
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float qs = amax > 0.0f ? 448.0f / amax : 1.0f;
    if (lane == 0) row_scale[r] = amax > 0.0f ? amax / 448.0f : 1.0f;
    uint2* out = reinterpret_cast<uint2*>(dst + r * cols);
    for (int v = lane; v < vecs; v += 32) {
      const uint4 u = row[v];
      const float2 a = unpack_bf16x2(u.x), b = unpack_bf16x2(u.y), c = unpack_bf16x2(u.z), d = unpack_bf16x2(u.w);
      const uint32_t lo = e4m3x2(a.x * qs, a.y * qs) | (e4m3x2(b.x * qs, b.y * qs) << 16);
      const uint32_t hi = e4m3x2(c.x * qs, c.y * qs) | (e4m3x2(d.x * qs, d.y * qs) << 16);
      out[v] = make_uint2(lo, hi);
    }
  }
}

// ------------------------------------------- tensor-parallel reduce-scatter
// Owner side: wait until every source published `epoch` (bounded), then
// out[i, j] = sum over s = 0..W-1 of recv[s, i, j] in that fixed order. W is
// a template argument so the W loads of an element are all issued before the
// adds (a loop over a run-time count kept one load in flight per thread).
template <typename OutT, int W>
__global__ void tp_reduce_rows_kernel(const float* __restrict__ recv, const uint32_t* flags, uint32_t epoch,
                                      OutT* __restrict__ out, long long rows, int n, uint32_t* status) {
  constexpr int world = W;
  __shared__ int ok;
  if (threadIdx.x == 0) {
    ok = 1;
    const uint64_t deadline = global_timer_ns() + 2ull * kWaitTimeoutNs;
    for (int s = 0; s < world; ++s) {
      const volatile uint32_t* f = flags + s;
      while (*f != epoch) {
        if (global_timer_ns() > deadline) {
          if (status) atomicOr(status, kErrTimeoutPeer);
          ok = 0;
          break;
        }
      }
      if (!ok) break;
    }
    __threadfence_system();
  }
  __syncthreads();
  if (!ok) return;
  const long long total4 = rows * (n / 4);
  const long long slab = rows * static_cast<long long>(n);
  for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < total4;
       e += (long long)gridDim.x * blockDim.x) {
    float4 v[W];
#pragma unroll
    for (int s = 0; s < W; ++s) v[s] = reinterpret_cast<const float4*>(recv + s * slab)[e];
    float4 acc = v[0];
#pragma unroll
    for (int s = 1; s < W; ++s) {
      acc.x += v[s].x;
      acc.y += v[s].y;
      acc.z += v[s].z;
      acc.w += v[s].w;
    }
    if constexpr (sizeof(OutT) == 4) {
      reinterpret_cast<float4*>(out)[e] = acc;
    } else {
      uint2 u;
      u.x = pack_bf16x2(acc.x, acc.y);
      u.y = pack_bf16x2(acc.z, acc.w);
      reinterpret_cast<uint2*>(out)[e] = u;
    }
  }
}

}  // namespace swiglu
