// Host side of the C ABI declared in include/swiglu_b200.h: argument checks,
// TMA tensor-map encoding, kernel selection and launch. No allocation: every
// buffer, including the per-stream stream-K workspace, is the caller's.
#include "swiglu_b200.h"

#include <cuda_runtime.h>

#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <mutex>
#include <string>

#include "simt_kernels.cuh"
#include "tc_dw2.cuh"
#include "tc_gemm2.cuh"

namespace swiglu {

// Bit mask of pipeline timeouts, one word per device (see ptx.cuh).
__device__ uint32_t g_status_word;

namespace {

thread_local std::string t_last_error;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  t_last_error = buf;
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(SWIGLU_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

constexpr int kMaxDevices = 64;
// Tile-order group (in 128-row tiles) for the GEMMs whose caller passes none:
// 32 (16 pair rows) measured at config 2 against 16: GEMM1 1.618 -> 1.590 ms
// with DRAM reads 1.87 -> 1.06 GB, y/dW1/dx within 0.2 %; walking every row
// tile per column band (88) doubled the DRAM reads (3.65 GB).
constexpr int kDefaultGroupM = 32;

struct DeviceInfo {
  std::atomic<bool> ready{false};
  int sms = 0;
  int major = 0;
  uint32_t* status = nullptr;
};

std::mutex g_mu;
DeviceInfo g_dev[kMaxDevices];

using CtxGetCurrentFn = CUresult (*)(CUcontext*);
using CtxGetDeviceFn = CUresult (*)(CUdevice*);

// The device an entry point works on is the device of the context bound to
// the calling thread (the one torch or any other runtime made current), so
// this library and its caller agree even though they link different CUDA
// runtimes. A thread that has never made a CUDA call (e.g. the autograd
// engine's device thread) has no context bound; driver calls such as
// cuTensorMapEncodeTiled would then fail with CUDA_ERROR_INVALID_CONTEXT, so
// the runtime's current device's primary context is bound first.
int resolve_device(int* out) {
  static CtxGetCurrentFn get_current = nullptr;
  static CtxGetDeviceFn get_device = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_current = reinterpret_cast<CtxGetCurrentFn>(p);
    if (cudaGetDriverEntryPoint("cuCtxGetDevice", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_device = reinterpret_cast<CtxGetDeviceFn>(p);
  });
  int rdev = 0;
  cudaError_t e = cudaGetDevice(&rdev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  CUcontext ctx = nullptr;
  CUdevice cdev = 0;
  if (get_current && get_device && get_current(&ctx) == CUDA_SUCCESS && ctx != nullptr &&
      get_device(&cdev) == CUDA_SUCCESS) {
    if (static_cast<int>(cdev) != rdev) {
      if ((e = cudaSetDevice(static_cast<int>(cdev))) != cudaSuccess) return cuda_fail(e, "cudaSetDevice");
    }
    *out = static_cast<int>(cdev);
    return SWIGLU_OK;
  }
  if ((e = cudaSetDevice(rdev)) != cudaSuccess) return cuda_fail(e, "cudaSetDevice");
  *out = rdev;
  return SWIGLU_OK;
}

int current_device(DeviceInfo** out) {
  int dev = 0;
  cudaError_t e = cudaSuccess;
  if (int rc = resolve_device(&dev)) return rc;
  if (dev < 0 || dev >= kMaxDevices) return fail(SWIGLU_ERR_UNSUPPORTED_DEVICE, "device ordinal %d out of range", dev);
  DeviceInfo& d = g_dev[dev];
  if (!d.ready.load(std::memory_order_acquire)) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (!d.ready.load(std::memory_order_relaxed)) {
      if ((e = cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess)
        return cuda_fail(e, "cudaDeviceGetAttribute(SM count)");
      if ((e = cudaDeviceGetAttribute(&d.major, cudaDevAttrComputeCapabilityMajor, dev)) != cudaSuccess)
        return cuda_fail(e, "cudaDeviceGetAttribute(CC major)");
      void* sym = nullptr;
      if ((e = cudaGetSymbolAddress(&sym, g_status_word)) != cudaSuccess)
        return cuda_fail(e, "cudaGetSymbolAddress(status word)");
      d.status = static_cast<uint32_t*>(sym);
      d.ready.store(true, std::memory_order_release);
    }
  }
  if (d.major != 10)
    return fail(SWIGLU_ERR_UNSUPPORTED_DEVICE, "device %d has compute capability %d.x; this library targets sm_100a",
                dev, d.major);
  *out = &d;
  return SWIGLU_OK;
}

// ------------------------------------------------------------ tensor maps
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

int get_encode_fn(EncodeTiledFn* out) {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  static cudaError_t err = cudaSuccess;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    err = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
    if (err == cudaSuccess && q == cudaDriverEntryPointSuccess) fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  if (!fn) return fail(SWIGLU_ERR_CUDA, "cuTensorMapEncodeTiled unavailable (%s)", cudaGetErrorName(err));
  *out = fn;
  return SWIGLU_OK;
}

// 2-D bf16 map over a row-major [outer, inner] view with row pitch `ld`
// elements; 128-byte swizzled boxes of {64, box_outer}.
int make_map(CUtensorMap* m, const void* ptr, uint64_t inner, uint64_t outer, uint64_t ld, uint32_t box_outer,
             const char* what) {
  EncodeTiledFn fn;
  if (int rc = get_encode_fn(&fn)) return rc;
  if (reinterpret_cast<uintptr_t>(ptr) % 16)
    return fail(SWIGLU_ERR_MISALIGNED, "%s: base address is not 16-byte aligned", what);
  if ((ld * 2) % 16)
    return fail(SWIGLU_ERR_MISALIGNED, "%s: row pitch of %llu elements is not a multiple of 8", what,
                (unsigned long long)ld);
  const cuuint64_t dims[2] = {inner, outer};
  const cuuint64_t strides[1] = {ld * 2};
  const cuuint32_t box[2] = {64, box_outer};
  const cuuint32_t es[2] = {1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, es,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(SWIGLU_ERR_CUDA, "%s: cuTensorMapEncodeTiled failed (CUresult %d)", what, (int)r);
  return SWIGLU_OK;
}

// Output map of a store GEMM: row-major [M, N] (pitch ld elements) in
// {32 x 32} boxes, 64-byte swizzle for bf16 rows of 64 bytes, 128-byte for f32.
int make_store_map(CUtensorMap* m, void* ptr, uint64_t N, uint64_t M, uint64_t ld, bool f32) {
  EncodeTiledFn fn;
  if (int rc = get_encode_fn(&fn)) return rc;
  const uint64_t es = f32 ? 4 : 2;
  if (reinterpret_cast<uintptr_t>(ptr) % 16) return fail(SWIGLU_ERR_MISALIGNED, "C: base address is not 16-byte aligned");
  if ((ld * es) % 16) return fail(SWIGLU_ERR_MISALIGNED, "C: row pitch is not a multiple of 16 bytes");
  const cuuint64_t dims[2] = {N, M};
  const cuuint64_t strides[1] = {ld * es};
  const cuuint32_t box[2] = {32, 32};
  const cuuint32_t elem[2] = {1, 1};
  CUresult r = fn(m, f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, ptr, dims, strides,
                  box, elem, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  f32 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(SWIGLU_ERR_CUDA, "C: cuTensorMapEncodeTiled failed (CUresult %d)", (int)r);
  return SWIGLU_OK;
}

// 4-D bf16 map gathering several 64-column blocks of a row-major matrix in
// one TMA operation: dims {64 columns, rows, blocks, groups} with byte
// strides {row pitch, 128 (next 64-column block), group_stride}; 128-byte
// swizzled boxes of {64, box_rows, 2, 2}, laid out in shared memory as
// [group][block][row][128 B] -- the layout four {64, box_rows} 2-D boxes at
// (c, c + 64, c + group_stride / 2, ...) give. The caller sizes `blocks` so
// that every in-range coordinate addresses bytes inside the row.
int make_map_gather4(CUtensorMap* m, const void* ptr, uint64_t rows, uint64_t ld_bytes, uint64_t blocks,
                     uint64_t group_stride, uint32_t box_rows, const char* what) {
  EncodeTiledFn fn;
  if (int rc = get_encode_fn(&fn)) return rc;
  if (reinterpret_cast<uintptr_t>(ptr) % 16 || ld_bytes % 16 || group_stride % 16)
    return fail(SWIGLU_ERR_MISALIGNED, "%s: base, row pitch and group stride must be 16-byte multiples", what);
  const cuuint64_t dims[4] = {64, rows, blocks, 2};
  const cuuint64_t strides[3] = {ld_bytes, 128, group_stride};
  const cuuint32_t box[4] = {64, box_rows, 2, 2};
  const cuuint32_t es[4] = {1, 1, 1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(ptr), dims, strides, box, es,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(SWIGLU_ERR_CUDA, "%s: cuTensorMapEncodeTiled failed (CUresult %d)", what, (int)r);
  return SWIGLU_OK;
}

// e4m3 operand map: row-major [rows, K] bytes, row pitch `ld` bytes; 128-byte
// swizzled boxes of {128 elements of K, box_rows rows}.
int make_map_e4m3(CUtensorMap* m, const void* ptr, uint64_t K, uint64_t rows, uint64_t ld, uint32_t box_rows,
                  const char* what) {
  EncodeTiledFn fn;
  if (int rc = get_encode_fn(&fn)) return rc;
  if (reinterpret_cast<uintptr_t>(ptr) % 16)
    return fail(SWIGLU_ERR_MISALIGNED, "%s: base address is not 16-byte aligned", what);
  if (ld % 16)
    return fail(SWIGLU_ERR_MISALIGNED, "%s: row pitch of %llu bytes is not a multiple of 16", what,
                (unsigned long long)ld);
  const cuuint64_t dims[2] = {K, rows};
  const cuuint64_t strides[1] = {ld};
  const cuuint32_t box[2] = {128, box_rows};
  const cuuint32_t es[2] = {1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(ptr), dims, strides, box, es,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(SWIGLU_ERR_CUDA, "%s: cuTensorMapEncodeTiled failed (CUresult %d)", what, (int)r);
  return SWIGLU_OK;
}

// Operand maps. K-major operand stored [rows][K]; MN-major stored [K][cols].
int map_kmajor(CUtensorMap* m, const void* p, int64_t rows, int64_t K, int64_t ld, uint32_t box_rows,
               const char* what) {
  return make_map(m, p, K, rows, ld, box_rows, what);
}
int map_mnmajor(CUtensorMap* m, const void* p, int64_t K, int64_t cols, int64_t ld, const char* what) {
  return make_map(m, p, cols, K, ld, 64, what);
}

// ------------------------------------------------------------ launching
constexpr uint32_t kMnLbo = 64 * 64 * 2;  // one {64, 64} bf16 box
constexpr uint32_t kMnSbo = 8 * 128;      // eight 128-byte swizzle rows

// GEMM kernel choice: 0 = by size, 1 = single-SM kernel, 2 = 2-SM kernel with
// 256 x 256 tiles, 3 = 2-SM kernel with 256 x 512 tiles.
std::atomic<int> g_gemm_path{0};

// SMs the persistent launches leave free (swiglu_b200_set_sm_reserve), so
// that kernels of other streams, e.g. NCCL collectives overlapped with the
// GEMMs, find SMs to run on.
std::atomic<int> g_sm_reserve{0};

// Per-kernel launch state: dynamic shared memory opt-in done (bit per device)
// and, for cluster kernels, how many CTA pairs fit at once on each device.
struct KernelState {
  std::atomic<uint64_t> ready{0};
  int max_clusters[kMaxDevices] = {};
};

template <auto Kernel>
KernelState& kernel_state() {
  static KernelState s;  // one per kernel function
  return s;
}

// Persistent single-CTA launch: one CTA per SM (at most one per tile).
template <auto kern, class Params>
int launch_single(const Params& p, int tiles, int threads, int smem, const DeviceInfo& d, cudaStream_t st,
                  const char* what) {
  KernelState& ks = kernel_state<kern>();
  int dev = 0;
  cudaGetDevice(&dev);
  if (!(ks.ready.load() & (1ull << dev))) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return cuda_fail(e, what);
    ks.ready.fetch_or(1ull << dev);
  }
  int sms = d.sms - g_sm_reserve.load(std::memory_order_relaxed);
  if (sms < 1) sms = 1;
  const int grid = tiles < sms ? tiles : sms;
  kern<<<grid, threads, smem, st>>>(p);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? SWIGLU_OK : cuda_fail(e, what);
}

cudaLaunchConfig_t pair_launch_config(cudaLaunchAttribute* attr, int threads, int smem, cudaStream_t st) {
  cudaLaunchConfig_t cfg = {};
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.blockDim = dim3(threads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cfg;
}

// How many CTA pairs of `kern` fit on the current device at once (queried
// once per device).
template <auto kern>
int pair_capacity(int threads, int smem, const DeviceInfo& d, int* out, const char* what) {
  KernelState& ks = kernel_state<kern>();
  int dev = 0;
  cudaGetDevice(&dev);
  if (!(ks.ready.load() & (1ull << dev))) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return cuda_fail(e, what);
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = pair_launch_config(attr, threads, smem, nullptr);
    cfg.gridDim = dim3(2 * (d.sms / 2));
    int n = 0;
    e = cudaOccupancyMaxActiveClusters(&n, kern, &cfg);
    if (e != cudaSuccess) return cuda_fail(e, what);
    if (n < 1) return fail(SWIGLU_ERR_CUDA, "%s: no CTA pair fits on device %d", what, dev);
    ks.max_clusters[dev] = n;
    ks.ready.fetch_or(1ull << dev);
  }
  const int keep = ks.max_clusters[dev] - (g_sm_reserve.load(std::memory_order_relaxed) + 1) / 2;
  *out = keep < 1 ? 1 : keep;
  return SWIGLU_OK;
}

// Persistent CTA-pair launch (clusters of 2): as many pairs as fit at once,
// at most one per work unit.
template <auto kern, class Params>
int launch_pair(const Params& p, int units, int threads, int smem, const DeviceInfo& d, cudaStream_t st,
                const char* what) {
  int cap = 0;
  if (int rc = pair_capacity<kern>(threads, smem, d, &cap, what)) return rc;
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = pair_launch_config(attr, threads, smem, st);
  cfg.gridDim = dim3(2 * (units < cap ? units : cap));
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, p);
  return e == cudaSuccess ? SWIGLU_OK : cuda_fail(e, what);
}

// ------------------------------------------------------------ stream-K workspaces
// A caller-owned device buffer per (device, stream), registered with
// swiglu_b200_set_stream_workspace. Layout: kSkCounterBytes of arrival
// counters (zero when registered; every launch leaves them zero), then the
// f32 partial tiles.
constexpr size_t kSkCounterBytes = 4096;
constexpr int kSkMaxSplit = 4;      // at most 4 parts per tail tile
constexpr int kSkMinBlocksPerPart = 4;

struct StreamWorkspace {
  int dev = -1;
  cudaStream_t stream = nullptr;
  uint8_t* ptr = nullptr;
  size_t bytes = 0;
  uint32_t epoch = 0;
};
constexpr int kMaxWorkspaces = 256;
std::mutex g_ws_mu;
StreamWorkspace g_ws[kMaxWorkspaces];

int set_workspace(void* ptr, size_t bytes, cudaStream_t st) {
  int dev = 0;
  if (int rc = resolve_device(&dev)) return rc;
  if (ptr && (reinterpret_cast<uintptr_t>(ptr) % 256))
    return fail(SWIGLU_ERR_MISALIGNED, "workspace must be 256-byte aligned");
  if (ptr && bytes < kSkCounterBytes)
    return fail(SWIGLU_ERR_INVALID_ARGUMENT, "workspace of %zu bytes is below the %zu-byte minimum", bytes,
                kSkCounterBytes);
  std::lock_guard<std::mutex> lk(g_ws_mu);
  StreamWorkspace* slot = nullptr;
  for (auto& w : g_ws) {
    if (w.ptr && w.dev == dev && w.stream == st) slot = &w;
  }
  if (!ptr) {
    if (slot) *slot = StreamWorkspace{};
    return SWIGLU_OK;
  }
  if (!slot) {
    for (auto& w : g_ws) {
      if (!w.ptr) {
        slot = &w;
        break;
      }
    }
  }
  if (!slot) return fail(SWIGLU_ERR_INVALID_ARGUMENT, "more than %d stream workspaces registered", kMaxWorkspaces);
  *slot = StreamWorkspace{dev, st, static_cast<uint8_t*>(ptr), bytes, slot->epoch};
  return SWIGLU_OK;
}

// The workspace of (current device, st) and a fresh epoch for one launch;
// false when none is registered.
bool take_workspace(cudaStream_t st, uint8_t** ptr, size_t* bytes, uint32_t* epoch) {
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lk(g_ws_mu);
  for (auto& w : g_ws) {
    if (w.ptr && w.dev == dev && w.stream == st) {
      w.epoch = w.epoch % 0xFFFFFFu + 1u;
      *ptr = w.ptr;
      *bytes = w.bytes;
      *epoch = w.epoch;
      return true;
    }
  }
  return false;
}

// Chooses the stream-K tail of a persistent launch of `tiles` tiles of
// `tile_floats` f32 accumulators on `clusters` pairs with `num_kb` K blocks:
// the tiles of the last, partial round are split into as many K ranges as
// there are idle pairs for (at most kSkMaxSplit, each of at least
// kSkMinBlocksPerPart blocks), if the stream has a workspace large enough.
// `slabs` arrival counters are used per tail tile.
void choose_stream_k(int tiles, int clusters, int num_kb, long long tile_floats, int slabs, cudaStream_t st,
                     float** partials, uint32_t** counters, int* tail_out, int* split_out, uint32_t* epoch_out) {
  *tail_out = 0;
  *split_out = 1;
  const int tail = tiles % clusters;
  if (tail == 0) return;
  // Only where the idle pairs of the last round are at least 5% of the
  // launch's pair-rounds: below that, the partial-tile traffic and the longer
  // epilogue of the finishing part cost about what the split wins (measured
  // at M=11136 on the grad_h GEMM: 2464 tiles, 2% idle, 2% slower split).
  const int rounds = (tiles + clusters - 1) / clusters;
  if ((clusters - tail) * 20 < clusters * rounds) return;
  int split = clusters / tail;
  if (split > kSkMaxSplit) split = kSkMaxSplit;
  if (split > num_kb / kSkMinBlocksPerPart) split = num_kb / kSkMinBlocksPerPart;
  if (split < 2) return;
  uint8_t* ws = nullptr;
  size_t bytes = 0;
  uint32_t epoch = 0;
  if (static_cast<size_t>(tail) * slabs * 4 > kSkCounterBytes) return;
  const size_t need = kSkCounterBytes + static_cast<size_t>(tail) * split * tile_floats * 4;
  if (!take_workspace(st, &ws, &bytes, &epoch) || bytes < need) return;
  *counters = reinterpret_cast<uint32_t*>(ws);
  *partials = reinterpret_cast<float*>(ws + kSkCounterBytes);
  *tail_out = tail;
  *split_out = split;
  *epoch_out = epoch;
}

template <class Cfg>
int launch_tc(TcParams& p, const DeviceInfo& d, cudaStream_t st) {
  p.mn_lbo = kMnLbo;
  p.mn_sbo = kMnSbo;
  p.status = d.status;
  return launch_single<tc_gemm_kernel<Cfg>>(p, p.tiles_m * p.tiles_n, Cfg::NUM_THREADS, Cfg::SMEM_BYTES, d, st,
                       "tcgen05 GEMM launch");
}

template <class Cfg>
int launch_tc2(TcParams& p, const DeviceInfo& d, cudaStream_t st) {
  constexpr auto kern = tc_gemm2_kernel<Cfg>;
  const char* what = "2-SM tcgen05 GEMM launch";
  p.mn_lbo = kMnLbo;
  p.mn_sbo = kMnSbo;
  p.status = d.status;
  int cap = 0;
  if (int rc = pair_capacity<kern>(Cfg::NUM_THREADS, Cfg::SMEM_BYTES, d, &cap, what)) return rc;
  const int tiles = p.tiles_m * p.tiles_n;
  // 8 slabs of 32 rows per 256-row tile: 4 epilogue warps in each CTA.
  choose_stream_k(tiles, cap, (p.K + Cfg::BK - 1) / Cfg::BK, static_cast<long long>(Cfg::BM) * Cfg::BN, 8, st,
                  &p.sk_partials, &p.sk_counters, &p.sk_tail, &p.sk_split, &p.sk_epoch);
  return launch_pair<kern>(p, tiles + p.sk_tail * (p.sk_split - 1), Cfg::NUM_THREADS, Cfg::SMEM_BYTES, d, st, what);
}

// Kernel family for one tcgen05 GEMM: 1 = single-SM (128-row tiles), 2 = CTA
// pair with 256 x 256 tiles, 3 = CTA pair with 256 x 512 tiles. `forced` is
// the process-wide path (0 = by size), `tiles_n` the output's 256-column
// tiles. By size, pairs pay off once there is at least one full wave of them.
// Plain-store GEMMs without a width preference take 256 x 512 tiles once
// those make 8 waves of pairs: at M=65536 D=8192 H=28672 (y: 55 waves,
// dW2: 24) they measured 17 % faster than 256 x 256 tiles at equal clocks,
// while at 4-5 waves (y and dW2 at M=11136 D=3584 H=14336) the 256-column
// tiles are faster. `wide_by_size` says whether the GEMM may take them by
// size at all: plain stores, and GEMM1 + SwiGLU (TMA epilogue) once its K is
// at least kSwigluWideMinK (below), and grad_h + dSwiGLU likewise.
int pick_gemm_mode(int64_t M, int64_t tiles_n, bool wide_by_size, int tile_n, int sms, int forced) {
  if (forced != 0) return forced;
  const int64_t tiles_m2 = (M + 255) / 256;
  const int64_t pairs = sms / 2;
  if (tiles_m2 * tiles_n < pairs) return 1;
  const bool wide = tile_n == 512 || (tile_n == 0 && wide_by_size && tiles_m2 * ((tiles_n + 1) / 2) >= 8 * pairs);
  return wide ? 3 : 2;
}

// GEMM1 + SwiGLU and grad_h + dSwiGLU (their TMA epilogues) take 256 x 512
// tiles by size (8 waves, as plain GEMMs) only from this K on. A 256 x 512
// tile fills TMEM, so its epilogue (three TMA boxes per chunk) overlaps the
// next tile's main loop by halves only, a cost that falls with K against the
// main loop; the wide tile reads a quarter fewer operand bytes per FLOP,
// which under the 1 kW power cap buys clock for the whole step. Measured at
// M=65536 D=8192 H=28672 (sustained, one B200, A/B in one call): the step
// with this rule 234.4-242.4 ms against 242.2-249.3 ms with GEMM1 and
// grad_h on 256 x 256; at M=11136 D=3584 H=14336 the narrow tiles win, in
// time and in energy per FLOP (GEMM1 1.85 vs 1.90 ms, grad_h 1.04 vs
// 1.16 ms under the cap).
constexpr int64_t kSwigluWideMinK = 8192;

// Runs one tcgen05 GEMM with epilogue EPI on the single-SM (128-row tiles) or
// the 2-SM (256-row tiles) kernel. p.tiles_n must be set; tiles_m is set here.
// `tile_n` is the caller's preference for the pair tile's width (256 or 512;
// 0 = by size, below); it applies where the size rule picks the 2-SM kernel
// and no path is forced with swiglu_b200_set_gemm_path.
template <bool A_MN, bool B_MN, int EPI, bool F32>
int run_gemm(TcParams& p, const DeviceInfo& d, cudaStream_t st, int tile_n = 0) {
  int mode = g_gemm_path.load(std::memory_order_relaxed);
  // The 2-SM dSwiGLU epilogue stores 32-column TMA boxes: whole chunks only.
  if (EPI == kEpiDswiglu && !(p.flags & kFlagTmaEpilogue)) mode = 1;
  const bool swiglu_tma = EPI == kEpiSwigluTma || (EPI == kEpiDswiglu && (p.flags & kFlagTmaEpilogue));
  mode = pick_gemm_mode(p.M, p.tiles_n, EPI == kEpiStore || (swiglu_tma && p.K >= kSwigluWideMinK), tile_n, d.sms,
                        mode);
  if (mode == 2 || mode == 3) {
    // group_m counts 128-row tiles (the reference's GROUP_SIZE_M,
    // fused_forward.py:58); a pair tile covers two of them.
    p.tiles_m = (p.M + 255) / 256;
    p.group_m = p.group_m > 1 ? p.group_m / 2 : 1;
    if (mode == 3) {  // 256 x 512 pair tiles: twice the columns per tile
      p.tiles_n = (p.tiles_n + 1) / 2;
      return launch_tc2<Tc2Cfg<A_MN, B_MN, EPI, F32, 2>>(p, d, st);
    }
    return launch_tc2<Tc2Cfg<A_MN, B_MN, EPI, F32>>(p, d, st);
  }
  p.tiles_m = (p.M + 127) / 128;
  // The single-SM kernel has the per-lane SwiGLU epilogue only.
  return launch_tc<TcCfg<256, A_MN, B_MN, EPI == kEpiSwigluTma ? kEpiSwiglu : EPI, F32>>(p, d, st);
}

// e4m3 GEMMs: always the 2-SM kernel (the single-SM kernel has no 8-bit
// path), 256 x 256 or 256 x 512 pair tiles by the same size rule.
template <int EPI, bool F32>
int run_gemm_e4m3(TcParams& p, const DeviceInfo& d, cudaStream_t st, int tile_n = 0) {
  int mode = g_gemm_path.load(std::memory_order_relaxed);
  mode = pick_gemm_mode(p.M, p.tiles_n, EPI == kEpiStore, tile_n, d.sms, mode == 1 ? 2 : mode);
  if (mode == 1) mode = 2;
  p.tiles_m = (p.M + 255) / 256;
  p.group_m = p.group_m > 1 ? p.group_m / 2 : 1;
  if (mode == 3) {
    p.tiles_n = (p.tiles_n + 1) / 2;
    return launch_tc2<Tc2Cfg<false, false, EPI, F32, 2, true>>(p, d, st);
  }
  return launch_tc2<Tc2Cfg<false, false, EPI, F32, 1, true>>(p, d, st);
}

template <bool A_MN, bool B_MN, int EPI, bool TRANSFORM>
int launch_simt(const SimtParams& p, int ntile_cols, cudaStream_t st) {
  dim3 grid(ntile_cols, (p.M + 63) / 64);
  if (grid.y > 65535) return fail(SWIGLU_ERR_INVALID_ARGUMENT, "M=%d too large for the fp32 path", p.M);
  simt_gemm_f32_kernel<A_MN, B_MN, EPI, TRANSFORM><<<grid, 256, 0, st>>>(p);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "fp32 GEMM launch");
  return SWIGLU_OK;
}

int pointwise_grid(long long work, const DeviceInfo& d) {
  long long g = (work + 255) / 256;
  const long long cap = static_cast<long long>(d.sms) * 16;
  if (g > cap) g = cap;
  return g < 1 ? 1 : static_cast<int>(g);
}

bool fits_int(int64_t v) { return v >= 0 && v <= 0x7fffffffLL; }

int check_dtype(int dtype) {
  if (dtype != SWIGLU_F32 && dtype != SWIGLU_BF16) return fail(SWIGLU_ERR_INVALID_ARGUMENT, "unknown dtype %d", dtype);
  return SWIGLU_OK;
}
int check_layout(int layout, int64_t H) {
  if (layout != SWIGLU_LAYOUT_STD && layout != SWIGLU_LAYOUT_PACKED128)
    return fail(SWIGLU_ERR_INVALID_ARGUMENT, "unknown layout %d", layout);
  if (layout == SWIGLU_LAYOUT_PACKED128 && H % kPackChunk)
    return fail(SWIGLU_ERR_INVALID_ARGUMENT, "packed layout needs H %% 128 == 0 (H=%lld)", (long long)H);
  return SWIGLU_OK;
}
int check_dims(const char* what, int64_t a, int64_t b, int64_t c) {
  if (!fits_int(a) || !fits_int(b) || !fits_int(c))
    return fail(SWIGLU_ERR_INVALID_ARGUMENT, "%s: dimensions must be in [0, 2^31)", what);
  return SWIGLU_OK;
}
int check_mult8(const char* what, int64_t v) {
  if (v % 8) return fail(SWIGLU_ERR_INVALID_ARGUMENT, "%s=%lld must be a multiple of 8", what, (long long)v);
  return SWIGLU_OK;
}

// ---------------------------------------------------------------- ops
int op_swiglu_fwd(const void* x, const void* w, void* preact, void* h, int64_t M, int64_t K, int64_t H, int dtype,
                  int w_form, int layout, int rounded, int group_m, cudaStream_t st) {
  if (int rc = check_dims("fused_matmul_swiglu_save_preact", M, K, 2 * H)) return rc;
  if (int rc = check_dtype(dtype)) return rc;
  if (int rc = check_layout(layout, H)) return rc;
  if (w_form != SWIGLU_W1_ROWS && w_form != SWIGLU_W1_T)
    return fail(SWIGLU_ERR_INVALID_ARGUMENT, "unknown w_form %d", w_form);
  if (w_form == SWIGLU_W1_ROWS && layout != SWIGLU_LAYOUT_STD)
    return fail(SWIGLU_ERR_INVALID_ARGUMENT, "the packed layout applies to the [D, 2H] weight form only");
  if (K <= 0 || H <= 0) return fail(SWIGLU_ERR_INVALID_ARGUMENT, "K and H must be positive");
  if (group_m < 1) return fail(SWIGLU_ERR_INVALID_ARGUMENT, "group_size_m must be >= 1");
  if (M == 0) return SWIGLU_OK;
  if (!x || !w || (!preact && !h)) return fail(SWIGLU_ERR_INVALID_ARGUMENT, "null pointer");
  DeviceInfo* d;
  if (int rc = current_device(&d)) return rc;
  if (dtype == SWIGLU_F32) {
    SimtParams p{};
    p.a = static_cast<const float*>(x);
    p.b = static_cast<const float*>(w);
    p.out0 = static_cast<float*>(preact);
    p.out1 = static_cast<float*>(h);
    p.lda = K;
    p.ldb = w_form == SWIGLU_W1_ROWS ? K : 2 * H;
    p.ld0 = 2 * H;
    p.ld1 = H;
    p.M = (int)M, p.N = (int)H, p.K = (int)K, p.H = (int)H, p.layout = layout;
    const int nt = (int)((H + 31) / 32);
    return w_form == SWIGLU_W1_ROWS ? launch_simt<false, false, kEpiSwiglu, false>(p, nt, st)
                                    : launch_simt<false, true, kEpiSwiglu, false>(p, nt, st);
  }
  if (int rc = check_mult8("K", K)) return rc;
  if (int rc = check_mult8("H", H)) return rc;
  TcParams p{};
  if (int rc = map_kmajor(&p.tmA, x, M, K, K, 128, "x")) return rc;
  if (w_form == SWIGLU_W1_ROWS) {
    if (int rc = map_kmajor(&p.tmB, w, 2 * H, K, K, 128, "W1")) return rc;
  } else {
    if (int rc = map_mnmajor(&p.tmB, w, K, 2 * H, 2 * H, "Wt")) return rc;
  }
  p.out0 = preact;
  p.out1 = h;
  p.ld0 = 2 * H;
  p.ld1 = H;
  p.M = (int)M, p.N = (int)H, p.K = (int)K, p.H = (int)H, p.layout = layout;
  p.tiles_n = (int)((H + 127) / 128);
  p.group_m = group_m;
  p.flags = rounded ? kFlagHFromRounded : 0;
  if ((preact && reinterpret_cast<uintptr_t>(preact) % 16) || (h && reinterpret_cast<uintptr_t>(h) % 16))
    return fail(SWIGLU_ERR_MISALIGNED, "preact/h must be 16-byte aligned");
  // The 2-SM kernel stores preact and h with TMA when every 32-unit chunk
  // below H is whole (its boxes are 32 columns wide) and M >= 4096: measured
  // on B200 at K=4096 H=14336, TMA stores take M=4096 from 0.668 to 0.653 ms
  // and config 2 from 1.604 to 1.569 ms, but M=1024 from 0.204 to 0.224 ms.
  if (H % 32 == 0 && M >= 4096) {
    if (preact) {
      if (int rc = make_store_map(&p.tmC, preact, 2 * H, M, 2 * H, false)) return rc;
    }
    if (h) {
      if (int rc = make_store_map(&p.tmD, h, H, M, H, false)) return rc;
    }
    return w_form == SWIGLU_W1_ROWS ? run_gemm<false, false, kEpiSwigluTma, false>(p, *d, st)
                                    : run_gemm<false, true, kEpiSwigluTma, false>(p, *d, st);
  }
  return w_form == SWIGLU_W1_ROWS ? run_gemm<false, false, kEpiSwiglu, false>(p, *d, st)
                                  : run_gemm<false, true, kEpiSwiglu, false>(p, *d, st);
}

int op_matmul(const void* a, const void* b, void* c, int64_t M, int64_t N, int64_t K, int a_layout, int b_layout,
              int dtype, int out_dtype, int group_m, cudaStream_t st, int tile_n = 0) {
  if (tile_n != 0 && tile_n != 256 && tile_n != 512)
    return fail(SWIGLU_ERR_INVALID_ARGUMENT, "tile_n must be 0, 256 or 512");
  if (int rc = check_dims("matmul", M, N, K)) return rc;
  if (int rc = check_dtype(dtype)) return rc;
  if (int rc = check_dtype(out_dtype)) return rc;
  if ((a_layout | b_layout) & ~1) return fail(SWIGLU_ERR_INVALID_ARGUMENT, "layout flags must be 0 or 1");
  if (dtype == SWIGLU_F32 && out_dtype != SWIGLU_F32)
    return fail(SWIGLU_ERR_INVALID_ARGUMENT, "an f32 GEMM writes f32");
  if (K <= 0) return fail(SWIGLU_ERR_INVALID_ARGUMENT, "K must be positive");
  if (group_m < 1) return fail(SWIGLU_ERR_INVALID_ARGUMENT, "group_size_m must be >= 1");
  if (M == 0 || N == 0) return SWIGLU_OK;
  if (!a || !b || !c) return fail(SWIGLU_ERR_INVALID_ARGUMENT, "null pointer");
  DeviceInfo* d;
  if (int rc = current_device(&d)) return rc;
  const bool a_mn = a_layout == 1;       // stored [K][M]
  const bool b_mn = b_layout == 0;       // stored [K][N]
  if (dtype == SWIGLU_F32) {
    SimtParams p{};
    p.a = static_cast<const float*>(a);
    p.b = static_cast<const float*>(b);
    p.out0 = static_cast<float*>(c);
    p.lda = a_mn ? M : K;
    p.ldb = b_mn ? N : K;
    p.ld0 = N;
    p.M = (int)M, p.N = (int)N, p.K = (int)K;
    const int nt = (int)((N + 63) / 64);
    if (a_mn) return b_mn ? launch_simt<true, true, kEpiStore, false>(p, nt, st)
                          : launch_simt<true, false, kEpiStore, false>(p, nt, st);
    return b_mn ? launch_simt<false, true, kEpiStore, false>(p, nt, st)
                : launch_simt<false, false, kEpiStore, false>(p, nt, st);
  }
  // TMA row pitches must be multiples of 16 bytes: the contiguous dimension of
  // each operand (K for a K-major operand, M or N for an MN-major one) and N
  // for the output rows.
  if (!a_mn || !b_mn) { if (int rc = check_mult8("K", K)) return rc; }
  if (a_mn) { if (int rc = check_mult8("M", M)) return rc; }
  if (int rc = check_mult8("N", N)) return rc;
  TcParams p{};
  if (a_mn) {
    if (int rc = map_mnmajor(&p.tmA, a, K, M, M, "A")) return rc;
  } else {
    if (int rc = map_kmajor(&p.tmA, a, M, K, K, 128, "A")) return rc;
  }
  if (b_mn) {
    if (int rc = map_mnmajor(&p.tmB, b, K, N, N, "B")) return rc;
  } else {
    if (int rc = map_kmajor(&p.tmB, b, N, K, K, 128, "B")) return rc;
  }
  if (reinterpret_cast<uintptr_t>(c) % 16) return fail(SWIGLU_ERR_MISALIGNED, "C must be 16-byte aligned");
  const bool f32 = out_dtype == SWIGLU_F32;
  if (int rc = make_store_map(&p.tmC, c, N, M, N, f32)) return rc;
  p.out0 = c;
  p.ld0 = N;
  p.M = (int)M, p.N = (int)N, p.K = (int)K, p.H = 0, p.layout = 0;
  p.tiles_n = (int)((N + 255) / 256);
  p.group_m = group_m;
#define SWIGLU_MM(AM, BM_, F) run_gemm<AM, BM_, kEpiStore, F>(p, *d, st, tile_n)
  if (f32) {
    if (a_mn) return b_mn ? SWIGLU_MM(true, true, true) : SWIGLU_MM(true, false, true);
    return b_mn ? SWIGLU_MM(false, true, true) : SWIGLU_MM(false, false, true);
  }
  if (a_mn) return b_mn ? SWIGLU_MM(true, true, false) : SWIGLU_MM(true, false, false);
  return b_mn ? SWIGLU_MM(false, true, false) : SWIGLU_MM(false, false, false);
#undef SWIGLU_MM
}

int op_matmul_scatter(const void* a, const void* b, int64_t M, int64_t N, int64_t K, int a_layout, int b_layout,
                      int dtype, void* const* peer_bufs, int world, int rank, int64_t rows_per_rank,
                      cudaStream_t st) {
  if (int rc = check_dims("matmul_scatter_rows", M, N, K)) return rc;
  if (dtype != SWIGLU_BF16) return fail(SWIGLU_ERR_INVALID_ARGUMENT, "the scatter GEMM takes bf16 operands");
  if ((a_layout | b_layout) & ~1) return fail(SWIGLU_ERR_INVALID_ARGUMENT, "layout flags must be 0 or 1");
  if (world < 1 || world > 8 || rank < 0 || rank >= world)
    return fail(SWIGLU_ERR_INVALID_ARGUMENT, "world must be 1..8 and 0 <= rank < world");
  if (rows_per_rank <= 0 || rows_per_rank * world != M)
    return fail(SWIGLU_ERR_INVALID_ARGUMENT, "M=%lld must equal world*rows_per_rank", (long long)M);
  if (K <= 0) return fail(SWIGLU_ERR_INVALID_ARGUMENT, "K must be positive");
  if (!a || !b || !peer_bufs) return fail(SWIGLU_ERR_INVALID_ARGUMENT, "null pointer");
  for (int i = 0; i < world; ++i) {
    if (!peer_bufs[i] || reinterpret_cast<uintptr_t>(peer_bufs[i]) % 16)
      return fail(SWIGLU_ERR_MISALIGNED, "peer buffer %d is null or not 16-byte aligned", i);
  }
  DeviceInfo* d;
  if (int rc = current_device(&d)) return rc;
  const bool a_mn = a_layout == 1, b_mn = b_layout == 0;
  if (!a_mn || !b_mn) { if (int rc = check_mult8("K", K)) return rc; }
  if (a_mn) { if (int rc = check_mult8("M", M)) return rc; }
  if (int rc = check_mult8("N", N)) return rc;
  TcParams p{};
  if (a_mn) {
    if (int rc = map_mnmajor(&p.tmA, a, K, M, M, "A")) return rc;
  } else {
    if (int rc = map_kmajor(&p.tmA, a, M, K, K, 128, "A")) return rc;
  }
  if (b_mn) {
    if (int rc = map_mnmajor(&p.tmB, b, K, N, N, "B")) return rc;
  } else {
    if (int rc = map_kmajor(&p.tmB, b, N, K, K, 128, "B")) return rc;
  }
  for (int i = 0; i < world; ++i) p.peer[i] = static_cast<float*>(peer_bufs[i]);
  p.rows_per_rank = (int)rows_per_rank;
  p.src_rank = rank;
  p.ld0 = N;
  p.M = (int)M, p.N = (int)N, p.K = (int)K;
  p.tiles_n = (int)((N + 255) / 256);
  p.group_m = kDefaultGroupM;
  if (a_mn) return b_mn ? run_gemm<true, true, kEpiScatterRows, true>(p, *d, st)
                        : run_gemm<true, false, kEpiScatterRows, true>(p, *d, st);
  return b_mn ? run_gemm<false, true, kEpiScatterRows, true>(p, *d, st)
              : run_gemm<false, false, kEpiScatterRows, true>(p, *d, st);
}

struct PeerFlags {
  uint32_t* f[8];
};

__global__ void tp_signal_param_kernel(PeerFlags pf, int world, int rank, uint32_t epoch) {
  const int o = threadIdx.x;
  if (o < world) {
    __threadfence_system();
    volatile uint32_t* f = pf.f[o] + rank;
    *f = epoch;
    __threadfence_system();
  }
}

int op_tp_signal(uint32_t* const* peer_flags, int world, int rank, uint32_t epoch, cudaStream_t st) {
  if (world < 1 || world > 8 || rank < 0 || rank >= world)
    return fail(SWIGLU_ERR_INVALID_ARGUMENT, "world must be 1..8 and 0 <= rank < world");
  if (!peer_flags) return fail(SWIGLU_ERR_INVALID_ARGUMENT, "null pointer");
  PeerFlags pf{};
  for (int i = 0; i < world; ++i) {
    if (!peer_flags[i]) return fail(SWIGLU_ERR_INVALID_ARGUMENT, "null flag pointer %d", i);
    pf.f[i] = peer_flags[i];
  }
  DeviceInfo* d;
  if (int rc = current_device(&d)) return rc;
  tp_signal_param_kernel<<<1, 32, 0, st>>>(pf, world, rank, epoch);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? SWIGLU_OK : cuda_fail(e, "tp_signal launch");
}

template <typename OutT>
void launch_tp_reduce(int world, int grid, cudaStream_t st, const float* recv, const uint32_t* flags, uint32_t epoch,
                      OutT* out, int64_t rows, int n, uint32_t* status) {
  switch (world) {
#define SWIGLU_TP_REDUCE_CASE(W) \
  case W: tp_reduce_rows_kernel<OutT, W><<<grid, 256, 0, st>>>(recv, flags, epoch, out, rows, n, status); break;
    SWIGLU_TP_REDUCE_CASE(1)
    SWIGLU_TP_REDUCE_CASE(2)
    SWIGLU_TP_REDUCE_CASE(3)
    SWIGLU_TP_REDUCE_CASE(4)
    SWIGLU_TP_REDUCE_CASE(5)
    SWIGLU_TP_REDUCE_CASE(6)
    SWIGLU_TP_REDUCE_CASE(7)
    SWIGLU_TP_REDUCE_CASE(8)
#undef SWIGLU_TP_REDUCE_CASE
    default: break;  // world is checked to be 1..8 by the caller
  }
}

int op_tp_reduce(const float* recv, const uint32_t* flags, int world, uint32_t epoch, void* out, int64_t rows,
                 int64_t N, int out_dtype, cudaStream_t st) {
  if (int rc = check_dims("tp_reduce_rows", rows, N, world)) return rc;
  if (world < 1 || world > 8) return fail(SWIGLU_ERR_INVALID_ARGUMENT, "world must be 1..8");
  if (int rc = check_dtype(out_dtype)) return rc;
  if (N % 4) return fail(SWIGLU_ERR_INVALID_ARGUMENT, "N=%lld must be a multiple of 4", (long long)N);
  if (!recv || !flags || !out) return fail(SWIGLU_ERR_INVALID_ARGUMENT, "null pointer");
  if (reinterpret_cast<uintptr_t>(recv) % 16 || reinterpret_cast<uintptr_t>(out) % 16)
    return fail(SWIGLU_ERR_MISALIGNED, "recv/out must be 16-byte aligned");
  DeviceInfo* d;
  if (int rc = current_device(&d)) return rc;
  if (rows == 0 || N == 0) return SWIGLU_OK;
  const int grid = pointwise_grid(rows * (N / 4), *d);
  if (out_dtype == SWIGLU_F32)
    launch_tp_reduce<float>(world, grid, st, recv, flags, epoch, static_cast<float*>(out), rows, (int)N, d->status);
  else
    launch_tp_reduce<__nv_bfloat16>(world, grid, st, recv, flags, epoch, static_cast<__nv_bfloat16*>(out), rows,
                                    (int)N, d->status);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? SWIGLU_OK : cuda_fail(e, "tp_reduce launch");
}

int op_dw2(const void* gy, const void* preact, void* dw2, int64_t M, int64_t H, int64_t Dout, int dtype, int layout,
           cudaStream_t st) {
  if (int rc = check_dims("bwd_dw2", M, 2 * H, Dout)) return rc;
  if (int rc = check_dtype(dtype)) return rc;
  if (int rc = check_layout(layout, H)) return rc;
  if (H <= 0 || Dout <= 0) return fail(SWIGLU_ERR_INVALID_ARGUMENT, "H and Dout must be positive");
  if (!dw2 || (M > 0 && (!gy || !preact))) return fail(SWIGLU_ERR_INVALID_ARGUMENT, "null pointer");
  DeviceInfo* d;
  if (int rc = current_device(&d)) return rc;
  if (M == 0) {
    cudaError_t e = cudaMemsetAsync(dw2, 0, Dout * H * (dtype == SWIGLU_F32 ? 4 : 2), st);
    return e == cudaSuccess ? SWIGLU_OK : cuda_fail(e, "cudaMemsetAsync(dW2)");
  }
  if (dtype == SWIGLU_F32) {
    SimtParams p{};
    p.a = static_cast<const float*>(gy);
    p.b = static_cast<const float*>(preact);
    p.out0 = static_cast<float*>(dw2);
    p.lda = Dout;
    p.ldb = 2 * H;
    p.ld0 = H;
    p.M = (int)Dout, p.N = (int)H, p.K = (int)M, p.H = (int)H, p.layout = layout;
    return launch_simt<true, true, kEpiStore, true>(p, (int)((H + 63) / 64), st);
  }
  if (int rc = check_mult8("H", H)) return rc;
  if (int rc = check_mult8("Dout", Dout)) return rc;
  Dw2Params p{};
  if (reinterpret_cast<uintptr_t>(dw2) % 16) return fail(SWIGLU_ERR_MISALIGNED, "dW2 must be 16-byte aligned");
  p.dw2 = static_cast<__nv_bfloat16*>(dw2);
  p.M = (int)M, p.H = (int)H, p.Dout = (int)Dout, p.layout = layout;
  p.tiles_d = (int)((Dout + Dw2Cfg::BD - 1) / Dw2Cfg::BD);
  p.status = d->status;
  const int pair_tiles = (int)((H + Dw2PairCfg::BJ - 1) / Dw2PairCfg::BJ) * p.tiles_d;
  int mode = g_gemm_path.load(std::memory_order_relaxed);
  if (mode == 0) mode = pair_tiles >= d->sms / 2 ? 2 : 1;
  if (mode >= 2) {
    p.tiles_j = (int)((H + Dw2PairCfg::BJ - 1) / Dw2PairCfg::BJ);
    const char* what = "dW2 (CTA pair)";
    // {64, BK} boxes of this kernel's stage height (the operands the 4-D
    // gathers below do not cover).
    if (int rc = make_map(&p.tm_pre, preact, 2 * H, M, 2 * H, Dw2PairCfg::BK, "preact")) return rc;
    if (int rc = make_map(&p.tm_gy, gy, Dout, M, Dout, Dw2PairCfg::BK, "grad_y")) return rc;
    // One TMA operation per stage for left/gate and one for grad_y where the
    // shapes keep every gathered block inside its row: left block b (of 64
    // units) and gate block b at +H columns (standard) or +128 (packed); the
    // grad_y halves 256 columns apart. A tile's left block index is at most
    // H/64 - 2 (standard) / 2H/64 - 4 (packed), its grad_y block at most
    // Dout/64 - 6, so `blocks` below admits every coordinate used and no
    // in-range coordinate reaches past the row.
    if (layout == SWIGLU_LAYOUT_STD ? H % 64 == 0 : H % 128 == 0) {
      const uint64_t blocks = layout == SWIGLU_LAYOUT_STD ? H / 64 : 2 * H / 64 - 2;
      const uint64_t gstride = layout == SWIGLU_LAYOUT_STD ? 2 * H : 256;
      if (int rc = make_map_gather4(&p.tm_lg4, preact, M, 4 * H, blocks, gstride, Dw2PairCfg::BK, "preact (4-D)"))
        return rc;
      p.gather |= 1;
    }
    if (Dout % 512 == 0) {
      if (int rc = make_map_gather4(&p.tm_gy4, gy, M, 2 * Dout, Dout / 64 - 4, 512, Dw2PairCfg::BK, "grad_y (4-D)"))
        return rc;
      p.gather |= 2;
    }
    if (int rc = make_store_map(&p.tm_out, dw2, H, Dout, H, false)) return rc;
    int cap = 0;
    if (int rc = pair_capacity<dw2_hprologue_pair_kernel>(Dw2PairCfg::NUM_THREADS, Dw2PairCfg::SMEM_BYTES, *d, &cap,
                                                         what))
      return rc;
    // 8 slabs of 32 hidden units per 256-unit tile: 4 epilogue warps per CTA.
    choose_stream_k(pair_tiles, cap, (int)((M + Dw2PairCfg::BK - 1) / Dw2PairCfg::BK),
                    static_cast<long long>(Dw2PairCfg::BJ) * Dw2PairCfg::BD, 8, st, &p.sk_partials, &p.sk_counters,
                    &p.sk_tail, &p.sk_split, &p.sk_epoch);
    return launch_pair<dw2_hprologue_pair_kernel>(p, pair_tiles + p.sk_tail * (p.sk_split - 1),
                                                  Dw2PairCfg::NUM_THREADS, Dw2PairCfg::SMEM_BYTES, *d, st, what);
  }
  p.tiles_j = (int)((H + Dw2Cfg::BJ - 1) / Dw2Cfg::BJ);
  if (int rc = make_map(&p.tm_pre, preact, 2 * H, M, 2 * H, Dw2Cfg::BK, "preact")) return rc;
  if (int rc = make_map(&p.tm_gy, gy, Dout, M, Dout, Dw2Cfg::BK, "grad_y")) return rc;
  return launch_single<dw2_hprologue_kernel>(p, p.tiles_j * p.tiles_d, Dw2Cfg::NUM_THREADS, Dw2Cfg::SMEM_BYTES,
                       *d, st, "dW2");
}

int op_fwd_logic(const void* preact, void* h, int64_t M, int64_t H, int dtype, int layout, cudaStream_t st);

// grad_preact in place of preact; with h non-NULL also h = swiglu(preact) of
// the values it replaced.
int op_grad_preact(const void* gy, const void* w2, void* preact, void* h, int64_t M, int64_t H, int64_t Dout,
                   int dtype, int layout, cudaStream_t st) {
  if (int rc = check_dims("bwd_grad_preact_inplace", M, 2 * H, Dout)) return rc;
  if (int rc = check_dtype(dtype)) return rc;
  if (int rc = check_layout(layout, H)) return rc;
  if (H <= 0 || Dout <= 0) return fail(SWIGLU_ERR_INVALID_ARGUMENT, "H and Dout must be positive");
  if (M == 0) return SWIGLU_OK;
  if (!gy || !w2 || !preact) return fail(SWIGLU_ERR_INVALID_ARGUMENT, "null pointer");
  DeviceInfo* d;
  if (int rc = current_device(&d)) return rc;
  if (dtype == SWIGLU_F32) {
    if (h) {  // fp32 correctness path: h first, from the preact about to be replaced
      if (int rc = op_fwd_logic(preact, h, M, H, dtype, layout, st)) return rc;
    }
    SimtParams p{};
    p.a = static_cast<const float*>(gy);
    p.b = static_cast<const float*>(w2);
    p.out0 = static_cast<float*>(preact);
    p.lda = Dout;
    p.ldb = H;
    p.ld0 = 2 * H;
    p.M = (int)M, p.N = (int)H, p.K = (int)Dout, p.H = (int)H, p.layout = layout;
    return launch_simt<false, true, kEpiDswiglu, false>(p, (int)((H + 63) / 64), st);
  }
  if (int rc = check_mult8("H", H)) return rc;
  if (int rc = check_mult8("Dout", Dout)) return rc;
  TcParams p{};
  if (int rc = map_kmajor(&p.tmA, gy, M, Dout, Dout, 128, "grad_y")) return rc;
  if (int rc = map_mnmajor(&p.tmB, w2, Dout, H, H, "W2")) return rc;
  if (reinterpret_cast<uintptr_t>(preact) % 16) return fail(SWIGLU_ERR_MISALIGNED, "preact must be 16-byte aligned");
  if (reinterpret_cast<uintptr_t>(h) % 16) return fail(SWIGLU_ERR_MISALIGNED, "h must be 16-byte aligned");
  p.out0 = preact;
  p.ld0 = 2 * H;
  p.out1 = h;
  p.ld1 = H;
  // The 2-SM kernel stores grad_preact and h with TMA when every 32-unit
  // chunk below H is whole (its boxes are 32 columns wide).
  if (H % 32 == 0) {
    if (int rc = make_store_map(&p.tmC, preact, 2 * H, M, 2 * H, false)) return rc;
    if (h) {
      if (int rc = make_store_map(&p.tmD, h, H, M, H, false)) return rc;
    }
    p.flags |= kFlagTmaEpilogue;
  }
  p.M = (int)M, p.N = (int)H, p.K = (int)Dout, p.H = (int)H, p.layout = layout;
  p.tiles_n = (int)((H + 255) / 256);
  p.group_m = kDefaultGroupM;
  return run_gemm<false, true, kEpiDswiglu, false>(p, *d, st);
}

int op_fwd_logic(const void* preact, void* h, int64_t M, int64_t H, int dtype, int layout, cudaStream_t st) {
  if (int rc = check_dims("forward_logic", M, 2 * H, 0)) return rc;
  if (int rc = check_dtype(dtype)) return rc;
  if (int rc = check_layout(layout, H)) return rc;
  if (int rc = check_mult8("H", H)) return rc;
  if (M == 0 || H == 0) return SWIGLU_OK;
  if (!preact || !h) return fail(SWIGLU_ERR_INVALID_ARGUMENT, "null pointer");
  if (reinterpret_cast<uintptr_t>(preact) % 16 || reinterpret_cast<uintptr_t>(h) % 16)
    return fail(SWIGLU_ERR_MISALIGNED, "preact/h must be 16-byte aligned");
  DeviceInfo* d;
  if (int rc = current_device(&d)) return rc;
  const int grid = pointwise_grid(M * (H / 8), *d);
  if (dtype == SWIGLU_F32)
    swiglu_fwd_pointwise_kernel<float><<<grid, 256, 0, st>>>((const float*)preact, (float*)h, M, (int)H, layout);
  else
    swiglu_fwd_pointwise_kernel<__nv_bfloat16>
        <<<grid, 256, 0, st>>>((const __nv_bfloat16*)preact, (__nv_bfloat16*)h, M, (int)H, layout);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? SWIGLU_OK : cuda_fail(e, "forward_logic launch");
}

int op_bwd_logic(const void* preact, const void* gh, void* gp, int64_t M, int64_t H, int dtype, int layout,
                 cudaStream_t st) {
  if (int rc = check_dims("backward_logic", M, 2 * H, 0)) return rc;
  if (int rc = check_dtype(dtype)) return rc;
  if (int rc = check_layout(layout, H)) return rc;
  if (int rc = check_mult8("H", H)) return rc;
  if (M == 0 || H == 0) return SWIGLU_OK;
  if (!preact || !gh || !gp) return fail(SWIGLU_ERR_INVALID_ARGUMENT, "null pointer");
  if (reinterpret_cast<uintptr_t>(preact) % 16 || reinterpret_cast<uintptr_t>(gh) % 16 ||
      reinterpret_cast<uintptr_t>(gp) % 16)
    return fail(SWIGLU_ERR_MISALIGNED, "buffers must be 16-byte aligned");
  DeviceInfo* d;
  if (int rc = current_device(&d)) return rc;
  const int grid = pointwise_grid(M * (H / 8), *d);
  if (dtype == SWIGLU_F32)
    swiglu_bwd_pointwise_kernel<float>
        <<<grid, 256, 0, st>>>((const float*)preact, (const float*)gh, (float*)gp, M, (int)H, layout);
  else
    swiglu_bwd_pointwise_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(
        (const __nv_bfloat16*)preact, (const __nv_bfloat16*)gh, (__nv_bfloat16*)gp, M, (int)H, layout);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? SWIGLU_OK : cuda_fail(e, "backward_logic launch");
}

int op_pack(const void* src, void* dst, int64_t K, int64_t Nh, int64_t B, int dtype, int unpack, cudaStream_t st) {
  if (int rc = check_dtype(dtype)) return rc;
  if (K < 0 || Nh < 0 || B <= 0) return fail(SWIGLU_ERR_INVALID_ARGUMENT, "bad pack dimensions");
  if (Nh % B) return fail(SWIGLU_ERR_INVALID_ARGUMENT, "N_half=%lld must be a multiple of block_n_half=%lld",
                          (long long)Nh, (long long)B);
  if (K == 0 || Nh == 0) return SWIGLU_OK;
  if (!src || !dst) return fail(SWIGLU_ERR_INVALID_ARGUMENT, "null pointer");
  if (src == dst) return fail(SWIGLU_ERR_INVALID_ARGUMENT, "pack source and destination must not alias");
  DeviceInfo* d;
  if (int rc = current_device(&d)) return rc;
  const int grid = pointwise_grid(K * 2 * Nh, *d);
  if (dtype == SWIGLU_F32)
    pack_chunked_kernel<float><<<grid, 256, 0, st>>>((const float*)src, (float*)dst, K, Nh, B, unpack);
  else
    pack_chunked_kernel<__nv_bfloat16>
        <<<grid, 256, 0, st>>>((const __nv_bfloat16*)src, (__nv_bfloat16*)dst, K, Nh, B, unpack);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? SWIGLU_OK : cuda_fail(e, "pack launch");
}

// ------------------------------------------------------------ e4m3 path
int op_quantize_e4m3(const void* src, void* dst, float* row_scale, int64_t rows, int64_t cols, int dtype,
                     cudaStream_t st) {
  if (int rc = check_dims("quantize_rows_e4m3", rows, cols, 0)) return rc;
  if (dtype != SWIGLU_BF16) return fail(SWIGLU_ERR_INVALID_ARGUMENT, "quantize_rows_e4m3 takes bf16 rows");
  if (int rc = check_mult8("cols", cols)) return rc;
  if (rows == 0 || cols == 0) return SWIGLU_OK;
  if (!src || !dst || !row_scale) return fail(SWIGLU_ERR_INVALID_ARGUMENT, "null pointer");
  if (reinterpret_cast<uintptr_t>(src) % 16 || reinterpret_cast<uintptr_t>(dst) % 8 ||
      reinterpret_cast<uintptr_t>(row_scale) % 4)
    return fail(SWIGLU_ERR_MISALIGNED, "src must be 16-byte, dst 8-byte and row_scale 4-byte aligned");
  DeviceInfo* d;
  if (int rc = current_device(&d)) return rc;
  long long blocks = (rows + 7) / 8;  // a warp per row, 8 warps per block
  const long long cap = static_cast<long long>(d->sms) * 16;
  if (blocks > cap) blocks = cap;
  quantize_rows_e4m3_kernel<<<static_cast<int>(blocks), 256, 0, st>>>(
      static_cast<const __nv_bfloat16*>(src), static_cast<uint8_t*>(dst), row_scale, rows, static_cast<int>(cols));
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? SWIGLU_OK : cuda_fail(e, "quantize_rows_e4m3 launch");
}

int op_swiglu_fwd_e4m3(const void* xq, const float* x_scale, const void* wq, const float* w_scale, void* preact,
                       void* h, int64_t M, int64_t K, int64_t H, int layout, int rounded, int group_m,
                       cudaStream_t st) {
  if (int rc = check_dims("fused_matmul_swiglu_e4m3", M, K, 2 * H)) return rc;
  if (int rc = check_layout(layout, H)) return rc;
  if (K <= 0 || H <= 0) return fail(SWIGLU_ERR_INVALID_ARGUMENT, "K and H must be positive");
  if (K % 16) return fail(SWIGLU_ERR_INVALID_ARGUMENT, "K=%lld must be a multiple of 16", (long long)K);
  if (H % 32) return fail(SWIGLU_ERR_INVALID_ARGUMENT, "H=%lld must be a multiple of 32", (long long)H);
  if (group_m < 1) return fail(SWIGLU_ERR_INVALID_ARGUMENT, "group_size_m must be >= 1");
  if (M == 0) return SWIGLU_OK;
  if (!xq || !x_scale || !wq || !w_scale || (!preact && !h))
    return fail(SWIGLU_ERR_INVALID_ARGUMENT, "null pointer");
  if ((preact && reinterpret_cast<uintptr_t>(preact) % 16) || (h && reinterpret_cast<uintptr_t>(h) % 16))
    return fail(SWIGLU_ERR_MISALIGNED, "preact/h must be 16-byte aligned");
  DeviceInfo* d;
  if (int rc = current_device(&d)) return rc;
  TcParams p{};
  if (int rc = make_map_e4m3(&p.tmA, xq, K, M, K, 128, "x (e4m3)")) return rc;
  if (int rc = make_map_e4m3(&p.tmB, wq, K, 2 * H, K, 128, "W1 (e4m3)")) return rc;
  if (preact) {
    if (int rc = make_store_map(&p.tmC, preact, 2 * H, M, 2 * H, false)) return rc;
  }
  if (h) {
    if (int rc = make_store_map(&p.tmD, h, H, M, H, false)) return rc;
  }
  p.out0 = preact;
  p.out1 = h;
  p.ld0 = 2 * H;
  p.ld1 = H;
  p.M = (int)M, p.N = (int)H, p.K = (int)K, p.H = (int)H, p.layout = layout;
  p.tiles_n = (int)((H + 127) / 128);
  p.group_m = group_m;
  p.flags = rounded ? kFlagHFromRounded : 0;
  p.scale_a = x_scale;
  p.scale_b = w_scale;
  return run_gemm_e4m3<kEpiSwigluTma, false>(p, *d, st);
}

int op_matmul_e4m3(const void* aq, const float* a_scale, const void* bq, const float* b_scale, void* c, int64_t M,
                   int64_t N, int64_t K, int out_dtype, int group_m, cudaStream_t st) {
  if (int rc = check_dims("matmul_e4m3", M, N, K)) return rc;
  if (int rc = check_dtype(out_dtype)) return rc;
  if (K <= 0) return fail(SWIGLU_ERR_INVALID_ARGUMENT, "K must be positive");
  if (K % 16) return fail(SWIGLU_ERR_INVALID_ARGUMENT, "K=%lld must be a multiple of 16", (long long)K);
  if (int rc = check_mult8("N", N)) return rc;
  if (group_m < 1) return fail(SWIGLU_ERR_INVALID_ARGUMENT, "group_size_m must be >= 1");
  if (M == 0 || N == 0) return SWIGLU_OK;
  if (!aq || !a_scale || !bq || !b_scale || !c) return fail(SWIGLU_ERR_INVALID_ARGUMENT, "null pointer");
  if (reinterpret_cast<uintptr_t>(c) % 16) return fail(SWIGLU_ERR_MISALIGNED, "C must be 16-byte aligned");
  DeviceInfo* d;
  if (int rc = current_device(&d)) return rc;
  TcParams p{};
  if (int rc = make_map_e4m3(&p.tmA, aq, K, M, K, 128, "A (e4m3)")) return rc;
  if (int rc = make_map_e4m3(&p.tmB, bq, K, N, K, 128, "B (e4m3)")) return rc;
  const bool f32 = out_dtype == SWIGLU_F32;
  if (int rc = make_store_map(&p.tmC, c, N, M, N, f32)) return rc;
  p.out0 = c;
  p.ld0 = N;
  p.M = (int)M, p.N = (int)N, p.K = (int)K;
  p.tiles_n = (int)((N + 255) / 256);
  p.group_m = group_m;
  p.scale_a = a_scale;
  p.scale_b = b_scale;
  return f32 ? run_gemm_e4m3<kEpiStore, true>(p, *d, st) : run_gemm_e4m3<kEpiStore, false>(p, *d, st);
}

// ------------------------------------------------ no-allocation variant
// The single-rank form of the fused reduce-scatter pipeline (scatter GEMM ->
// signal -> reduce) with its receive buffer and flags in file-scope device
// arrays instead of caller memory. The arrays live on every GPU that loads
// this library until the process exits; every call shares them.
constexpr long long kNoAllocScratchFloats = 4ll << 20;  // 16 MiB of f32: M * N <= 4,194,304
static __device__ __align__(256) float g_noalloc_scratch[kNoAllocScratchFloats];
static __device__ __align__(256) uint32_t g_noalloc_flags[8];

struct NoAllocState {
  std::atomic<bool> ready{false};
  float* scratch = nullptr;
  uint32_t* flags = nullptr;
  std::atomic<uint32_t> epoch{0};
};
NoAllocState g_noalloc[kMaxDevices];

int op_matmul_reduce_noalloc(const void* a, const void* b, void* out, int64_t M, int64_t N, int64_t K,
                             int a_layout, int b_layout, int out_dtype, cudaStream_t st) {
  if (int rc = check_dims("matmul_reduce_rows_noalloc", M, N, K)) return rc;
  if (M * N > kNoAllocScratchFloats)
    return fail(SWIGLU_ERR_INVALID_ARGUMENT,
                "matmul_reduce_rows_noalloc: M*N=%lld exceeds the static scratch of %lld floats (16 MiB)",
                (long long)(M * N), kNoAllocScratchFloats);
  if (M == 0 || N == 0) return SWIGLU_OK;
  if (!out) return fail(SWIGLU_ERR_INVALID_ARGUMENT, "null pointer");
  DeviceInfo* d;
  if (int rc = current_device(&d)) return rc;
  int dev = 0;
  cudaGetDevice(&dev);
  NoAllocState& s = g_noalloc[dev];
  if (!s.ready.load(std::memory_order_acquire)) {
    // Set-up, once per device, with that device current: resolve the device
    // addresses of the static arrays (their host-side names are not device
    // addresses).
    std::lock_guard<std::mutex> lk(g_mu);
    if (!s.ready.load(std::memory_order_relaxed)) {
      void* p = nullptr;
      cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
      if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(no-alloc scratch)");
      s.scratch = static_cast<float*>(p);
      e = cudaGetSymbolAddress(&p, g_noalloc_flags);
      if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(no-alloc flags)");
      s.flags = static_cast<uint32_t*>(p);
      s.ready.store(true, std::memory_order_release);
    }
  }
  // The flags keep the previous call's value; a fresh epoch per call means
  // nothing has to be cleared (the GEMM overwrites all M*N scratch floats).
  uint32_t epoch = s.epoch.fetch_add(1) + 1;
  if (epoch == 0) epoch = s.epoch.fetch_add(1) + 1;
  void* peers[1] = {s.scratch};
  if (int rc = op_matmul_scatter(a, b, M, N, K, a_layout, b_layout, SWIGLU_BF16, peers, 1, 0, M, st)) return rc;
  uint32_t* flag_ptrs[1] = {s.flags};
  if (int rc = op_tp_signal(flag_ptrs, 1, 0, epoch, st)) return rc;
  return op_tp_reduce(s.scratch, s.flags, 1, epoch, out, M, N, out_dtype, st);
}

}  // namespace
}  // namespace swiglu

using namespace swiglu;

extern "C" {

int swiglu_b200_abi_version(void) { return SWIGLU_B200_ABI_VERSION; }

const char* swiglu_b200_status_string(int status) {
  switch (status) {
    case SWIGLU_OK: return "SWIGLU_OK";
    case SWIGLU_ERR_INVALID_ARGUMENT: return "SWIGLU_ERR_INVALID_ARGUMENT";
    case SWIGLU_ERR_MISALIGNED: return "SWIGLU_ERR_MISALIGNED";
    case SWIGLU_ERR_UNSUPPORTED_DEVICE: return "SWIGLU_ERR_UNSUPPORTED_DEVICE";
    case SWIGLU_ERR_CUDA: return "SWIGLU_ERR_CUDA";
    case SWIGLU_ERR_DEVICE_TIMEOUT: return "SWIGLU_ERR_DEVICE_TIMEOUT";
    default: return "SWIGLU_ERR_UNKNOWN";
  }
}

const char* swiglu_b200_last_error_message(void) { return t_last_error.c_str(); }

int swiglu_b200_device_status(uint32_t* bits, int clear) {
  if (!bits) return fail(SWIGLU_ERR_INVALID_ARGUMENT, "null pointer");
  DeviceInfo* d;
  if (int rc = current_device(&d)) return rc;
  uint32_t v = 0;
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceSynchronize");
  e = cudaMemcpy(&v, d->status, sizeof(v), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return cuda_fail(e, "read status word");
  if (clear) {
    e = cudaMemset(d->status, 0, sizeof(uint32_t));
    if (e != cudaSuccess) return cuda_fail(e, "clear status word");
  }
  *bits = v;
  return v ? fail(SWIGLU_ERR_DEVICE_TIMEOUT, "kernel pipeline wait timed out (bits 0x%x)", v) : SWIGLU_OK;
}

int swiglu_b200_matmul_scatter_rows(const void* a, const void* b, int64_t M, int64_t N, int64_t K, int a_layout,
                                    int b_layout, int dtype, void* const* peer_bufs, int world, int rank,
                                    int64_t rows_per_rank, void* stream) {
  return op_matmul_scatter(a, b, M, N, K, a_layout, b_layout, dtype, peer_bufs, world, rank, rows_per_rank,
                           static_cast<cudaStream_t>(stream));
}

int swiglu_b200_tp_signal(uint32_t* const* peer_flags, int world, int rank, uint32_t epoch, void* stream) {
  return op_tp_signal(peer_flags, world, rank, epoch, static_cast<cudaStream_t>(stream));
}

int swiglu_b200_tp_reduce_rows(const float* recv, const uint32_t* flags, int world, uint32_t epoch, void* out,
                               int64_t rows, int64_t N, int out_dtype, void* stream) {
  return op_tp_reduce(recv, flags, world, epoch, out, rows, N, out_dtype, static_cast<cudaStream_t>(stream));
}

int swiglu_b200_matmul_reduce_rows_noalloc(const void* a, const void* b, void* out, int64_t M, int64_t N,
                                           int64_t K, int a_layout, int b_layout, int out_dtype, void* stream) {
  return op_matmul_reduce_noalloc(a, b, out, M, N, K, a_layout, b_layout, out_dtype,
                                  static_cast<cudaStream_t>(stream));
}

int swiglu_b200_set_stream_workspace(void* workspace, size_t bytes, void* stream) {
  return set_workspace(workspace, bytes, static_cast<cudaStream_t>(stream));
}

int swiglu_b200_gemm_plan(int64_t M, int64_t N, int tile_n, int num_sms, int* family) {
  if (!family) return fail(SWIGLU_ERR_INVALID_ARGUMENT, "null pointer");
  if (tile_n != 0 && tile_n != 256 && tile_n != 512)
    return fail(SWIGLU_ERR_INVALID_ARGUMENT, "tile_n must be 0, 256 or 512");
  if (int rc = check_dims("gemm_plan", M, N, 1)) return rc;
  if (num_sms < 2) return fail(SWIGLU_ERR_INVALID_ARGUMENT, "num_sms must be >= 2");
  *family = pick_gemm_mode(M, (N + 255) / 256, true, tile_n, num_sms, g_gemm_path.load(std::memory_order_relaxed));
  return SWIGLU_OK;
}

int swiglu_b200_swiglu_fwd_plan(int64_t M, int64_t K, int64_t H, int num_sms, int* family) {
  if (!family) return fail(SWIGLU_ERR_INVALID_ARGUMENT, "null pointer");
  if (int rc = check_dims("swiglu_fwd_plan", M, K, 2 * H)) return rc;
  if (num_sms < 2) return fail(SWIGLU_ERR_INVALID_ARGUMENT, "num_sms must be >= 2");
  *family = pick_gemm_mode(M, (2 * H + 255) / 256, K >= kSwigluWideMinK, 0, num_sms,
                           g_gemm_path.load(std::memory_order_relaxed));
  return SWIGLU_OK;
}

int swiglu_b200_set_sm_reserve(int sms) {
  if (sms < 0 || sms > 64) return fail(SWIGLU_ERR_INVALID_ARGUMENT, "SM reserve must be in [0, 64]");
  g_sm_reserve.store(sms);
  return SWIGLU_OK;
}

int swiglu_b200_set_gemm_path(int mode) {
  if (mode < 0 || mode > 3) return fail(SWIGLU_ERR_INVALID_ARGUMENT, "gemm path must be 0, 1, 2 or 3");
  g_gemm_path.store(mode);
  return SWIGLU_OK;
}

int swiglu_b200_fused_matmul_swiglu_save_preact(const void* x, const void* w, void* preact, void* h, int64_t M,
                                                int64_t K, int64_t H, int dtype, int w_form, int layout,
                                                int h_from_rounded_preact, int group_size_m, void* stream) {
  return op_swiglu_fwd(x, w, preact, h, M, K, H, dtype, w_form, layout, h_from_rounded_preact, group_size_m,
                       static_cast<cudaStream_t>(stream));
}

int swiglu_b200_matmul(const void* a, const void* b, void* c, int64_t M, int64_t N, int64_t K, int a_layout,
                       int b_layout, int dtype, int out_dtype, int group_size_m, void* stream) {
  return op_matmul(a, b, c, M, N, K, a_layout, b_layout, dtype, out_dtype, group_size_m,
                   static_cast<cudaStream_t>(stream));
}

int swiglu_b200_matmul_tiled(const void* a, const void* b, void* c, int64_t M, int64_t N, int64_t K, int a_layout,
                             int b_layout, int dtype, int out_dtype, int group_size_m, int tile_n, void* stream) {
  return op_matmul(a, b, c, M, N, K, a_layout, b_layout, dtype, out_dtype, group_size_m,
                   static_cast<cudaStream_t>(stream), tile_n);
}

int swiglu_b200_bwd_dw2(const void* grad_y, const void* preact, void* dw2, int64_t M, int64_t H, int64_t Dout,
                        int dtype, int layout, void* stream) {
  return op_dw2(grad_y, preact, dw2, M, H, Dout, dtype, layout, static_cast<cudaStream_t>(stream));
}

int swiglu_b200_bwd_grad_preact_inplace(const void* grad_y, const void* w2, void* preact, int64_t M, int64_t H,
                                        int64_t Dout, int dtype, int layout, void* stream) {
  return op_grad_preact(grad_y, w2, preact, nullptr, M, H, Dout, dtype, layout, static_cast<cudaStream_t>(stream));
}

int swiglu_b200_bwd_grad_preact_inplace_emit_h(const void* grad_y, const void* w2, void* preact, void* h, int64_t M,
                                               int64_t H, int64_t Dout, int dtype, int layout, void* stream) {
  if (M > 0 && !h) return fail(SWIGLU_ERR_INVALID_ARGUMENT, "null pointer");
  return op_grad_preact(grad_y, w2, preact, h, M, H, Dout, dtype, layout, static_cast<cudaStream_t>(stream));
}

int swiglu_b200_forward_logic(const void* preact, void* h, int64_t M, int64_t H, int dtype, int layout,
                              void* stream) {
  return op_fwd_logic(preact, h, M, H, dtype, layout, static_cast<cudaStream_t>(stream));
}

int swiglu_b200_backward_logic(const void* preact, const void* grad_h, void* grad_preact, int64_t M, int64_t H,
                               int dtype, int layout, void* stream) {
  return op_bwd_logic(preact, grad_h, grad_preact, M, H, dtype, layout, static_cast<cudaStream_t>(stream));
}

int swiglu_b200_pack_weight_chunked(const void* src, void* dst, int64_t K, int64_t N_half, int64_t block_n_half,
                                    int dtype, int unpack, void* stream) {
  return op_pack(src, dst, K, N_half, block_n_half, dtype, unpack, static_cast<cudaStream_t>(stream));
}

int swiglu_b200_quantize_rows_e4m3(const void* src, void* dst, float* row_scale, int64_t rows, int64_t cols,
                                   int dtype, void* stream) {
  return op_quantize_e4m3(src, dst, row_scale, rows, cols, dtype, static_cast<cudaStream_t>(stream));
}

int swiglu_b200_fused_matmul_swiglu_e4m3(const void* xq, const float* x_scale, const void* w1q, const float* w1_scale,
                                         void* preact, void* h, int64_t M, int64_t K, int64_t H, int layout,
                                         int h_from_rounded_preact, int group_size_m, void* stream) {
  return op_swiglu_fwd_e4m3(xq, x_scale, w1q, w1_scale, preact, h, M, K, H, layout, h_from_rounded_preact,
                            group_size_m, static_cast<cudaStream_t>(stream));
}

int swiglu_b200_matmul_e4m3(const void* aq, const float* a_scale, const void* bq, const float* b_scale, void* c,
                            int64_t M, int64_t N, int64_t K, int out_dtype, int group_size_m, void* stream) {
  return op_matmul_e4m3(aq, a_scale, bq, b_scale, c, M, N, K, out_dtype, group_size_m,
                        static_cast<cudaStream_t>(stream));
}

int swiglu_b200_mlp_forward(const void* x, const void* w1, const void* w2, void* preact, void* h_workspace,
                            void* y, int64_t M, int64_t D, int64_t H, int64_t Dout, int dtype, int w_form,
                            int layout, int h_from_rounded_preact, void* stream) {
  if (M > 0 && (!h_workspace || !y || !w2)) return fail(SWIGLU_ERR_INVALID_ARGUMENT, "null pointer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (int rc = op_swiglu_fwd(x, w1, preact, h_workspace, M, D, H, dtype, w_form, layout, h_from_rounded_preact, 16,
                             st))
    return rc;
  // y [M, Dout] = h [M, H] . W2^T, W2 stored [Dout, H] (swiglu_recompute.py:65)
  return op_matmul(h_workspace, w2, y, M, Dout, H, 0, 1, dtype, dtype, 16, st);
}

int swiglu_b200_mlp_backward(const void* x, const void* w1, const void* w2, void* preact, const void* grad_y,
                             void* dx, void* dw1, void* dw2, int64_t M, int64_t D, int64_t H, int64_t Dout,
                             int dtype, int w_form, int layout, void* stream) {
  if (!w1 || !dw1 || (M > 0 && (!x || !dx))) return fail(SWIGLU_ERR_INVALID_ARGUMENT, "null pointer");
  if (w_form != SWIGLU_W1_ROWS && w_form != SWIGLU_W1_T)
    return fail(SWIGLU_ERR_INVALID_ARGUMENT, "unknown w_form %d", w_form);
  if (w_form == SWIGLU_W1_ROWS && layout != SWIGLU_LAYOUT_STD)
    return fail(SWIGLU_ERR_INVALID_ARGUMENT, "the packed layout applies to the [D, 2H] weight form only");
  if (int rc = check_dims("mlp_backward", M, D, 2 * H)) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // dW2 reads preact, so it runs before grad_preact overwrites it.
  if (int rc = op_dw2(grad_y, preact, dw2, M, H, Dout, dtype, layout, st)) return rc;
  if (int rc = op_grad_preact(grad_y, w2, preact, nullptr, M, H, Dout, dtype, layout, st)) return rc;
  if (M == 0) {
    const size_t es = dtype == SWIGLU_F32 ? 4 : 2;
    cudaError_t e = cudaMemsetAsync(dw1, 0, (size_t)(2 * H * D) * es, st);
    return e == cudaSuccess ? SWIGLU_OK : cuda_fail(e, "cudaMemsetAsync(dW1)");
  }
  if (w_form == SWIGLU_W1_ROWS) {
    // grad_W1 [2H, D] = grad_preact^T . x (swiglu_recompute.py:76)
    if (int rc = op_matmul(preact, x, dw1, 2 * H, D, M, 1, 0, dtype, dtype, 16, st, 512)) return rc;
    // grad_x [M, D] = grad_preact . W1, W1 stored [2H, D] (swiglu_recompute.py:77)
    return op_matmul(preact, w1, dx, M, D, 2 * H, 0, 0, dtype, dtype, 16, st, 512);
  }
  // grad_wt [D, 2H] = x^T . grad_preact (fused_forward.py:282)
  if (int rc = op_matmul(x, preact, dw1, D, 2 * H, M, 1, 0, dtype, dtype, 16, st, 512)) return rc;
  // grad_x [M, D] = grad_preact . wt^T, wt stored [D, 2H] (fused_forward.py:283)
  return op_matmul(preact, w1, dx, M, D, 2 * H, 0, 1, dtype, dtype, 16, st, 512);
}

}  // extern "C"
