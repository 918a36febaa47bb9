/*
 * swiglu_b200.h - C ABI of the B200 (sm_100a) SwiGLU-MLP recompute hot path.
 *
 * Plain pointers, sizes and enums only: no framework types cross this
 * boundary. Every tensor is dense, row-major and contiguous; every pointer is
 * device memory on the CURRENT CUDA device; `stream` is a cudaStream_t (NULL =
 * legacy default stream). All work is enqueued asynchronously on `stream`;
 * no entry point allocates device memory (outputs and workspaces are owned
 * and passed in by the caller).
 *
 * Shapes follow the reference (swiglu_recompute.py:12-13):
 *   x [M, D]   W1 [2H, D]  (or Wt = W1^T [D, 2H], standard or packed)
 *   W2 [Dout, H]   preact [M, 2H]   h [M, H]   y [M, Dout]
 *
 * Reference citations are file:line inside tongzhou8086/swiglu-recompute.
 * The reference is Python; each entry point below is the native replacement
 * of the Python function cited beside it.
 */
#ifndef SWIGLU_B200_H
#define SWIGLU_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SWIGLU_B200_ABI_VERSION 1

/* Status codes returned by every entry point. */
enum swiglu_status {
  SWIGLU_OK = 0,
  SWIGLU_ERR_INVALID_ARGUMENT = 1,   /* a shape/dtype/layout precondition failed (the reference's AssertionError) */
  SWIGLU_ERR_MISALIGNED = 2,         /* pointer or row pitch not 16-byte aligned (TMA requirement) */
  SWIGLU_ERR_UNSUPPORTED_DEVICE = 3, /* current device is not compute capability 10.x (B200) */
  SWIGLU_ERR_CUDA = 4,               /* a CUDA runtime or driver call failed */
  SWIGLU_ERR_DEVICE_TIMEOUT = 5      /* a kernel's bounded pipeline wait expired (see swiglu_b200_device_status) */
};

/* Element types. */
enum swiglu_dtype { SWIGLU_F32 = 0, SWIGLU_BF16 = 1 };

/* Column layout of preact / the first-layer weight over its 2H axis.
 * STD: [left | gate] (swiglu_recompute.py:29).
 * PACKED128: [left0|gate0|left1|gate1|...] in 128-column chunks
 *            (fused_forward_packed.py:77-92, BLOCK_SIZE_N_HALF = 128). */
enum swiglu_layout { SWIGLU_LAYOUT_STD = 0, SWIGLU_LAYOUT_PACKED128 = 1 };

/* Storage form of the first-layer weight.
 * ROWS: W1 [2H, D], the nn.Linear layout of SwiGLUMLPCustom (swiglu_recompute.py:92).
 * T:    W1^T [D, 2H]: `w1t` of SwiGLUMLPFused (fused_forward.py:299) or
 *       `packed_weight` of SwiGLUMLPPackedFused (fused_forward_packed.py:331). */
enum swiglu_w1_form { SWIGLU_W1_ROWS = 0, SWIGLU_W1_T = 1 };

/* ABI version of the loaded library (== SWIGLU_B200_ABI_VERSION). */
int swiglu_b200_abi_version(void);

/* Human-readable name of a status code. */
const char* swiglu_b200_status_string(int status);

/* Detail of the last failing call on this host thread ("" if none). */
const char* swiglu_b200_last_error_message(void);

/* Reads (and optionally clears) the device status word of the current device:
 * a bit mask of kernel pipeline timeouts. Synchronises the device. 0 = healthy. */
int swiglu_b200_device_status(uint32_t* bits, int clear);

/* Selects the tcgen05 GEMM kernel family for subsequent calls (process-wide):
 * 0 = by problem size (default), 1 = single-SM kernel (128-row tiles),
 * 2 = 2-SM kernel (cta_group::2, 256 x 256 tiles on a CTA pair),
 * 3 = 2-SM kernel with 256 x 512 tiles (one accumulator filling TMEM).
 * The dW2 prologue kernel has no 256 x 512 form (3 selects its 2-SM kernel).
 * Results are identical up to f32 summation order; this exists for testing
 * and tuning. No reference counterpart (the reference's Triton kernels pick
 * their tiling at compile time, fused_forward.py:55-65). */
int swiglu_b200_set_gemm_path(int mode);

/* Number of SMs (0..64, default 0) that the persistent GEMM launches leave
 * free from now on (process-wide): a launch then holds at most
 * (SMs - sms) / 2 CTA pairs (or SMs - sms single CTAs), so kernels on other
 * streams -- a collective overlapped with the GEMMs, for instance -- are not
 * kept waiting for the GEMM's last CTA. Results are unchanged. No reference
 * counterpart (single-GPU, one stream). */
int swiglu_b200_set_sm_reserve(int sms);

/* The kernel family swiglu_b200_matmul_tiled would run a bf16 GEMM with an
 * [M, N] output on, for a device with `num_sms` SMs: *family = 1 (single-SM),
 * 2 (CTA pair, 256 x 256 tiles) or 3 (CTA pair, 256 x 512 tiles), honouring a
 * path forced with swiglu_b200_set_gemm_path. Host-only (no device call). No
 * reference counterpart (Triton autotuning picks tiles inside the launch,
 * fused_forward.py:55-65). */
int swiglu_b200_gemm_plan(int64_t M, int64_t N, int tile_n, int num_sms, int* family);

/* The same for the bf16 GEMM1 + SwiGLU forward of swiglu_b200_fused_matmul_
 * swiglu_save_preact at M tokens, K = D inputs and H hidden units (the
 * [M, 2H] preact tiled by the pair kernels' TMA epilogue): 256 x 512 tiles by
 * size only from K >= 8192. Host-only. No reference counterpart (Triton
 * autotuning, fused_forward.py:55-65). */
int swiglu_b200_swiglu_fwd_plan(int64_t M, int64_t K, int64_t H, int num_sms, int* family);

/* Recommended size of a stream-K workspace (48 MiB). */
#define SWIGLU_B200_STREAM_WORKSPACE_BYTES ((size_t)48 << 20)

/* Registers `workspace` (device memory of the current device, 256-byte
 * aligned, `bytes` >= 4096, the first 4096 bytes zero-filled) for GEMMs
 * launched on `stream`; NULL unregisters. With a workspace, the 2-SM GEMM
 * kernels split the tiles of their last, partial round of CTA pairs along K
 * (stream-K), so every pair stays busy to the end; the parts are added in a
 * fixed order, so results are run-to-run identical, but differ from the
 * unsplit kernel in f32 summation order. Without one (or one too small for a
 * launch) the unsplit kernel runs. Launches on one stream share its
 * workspace in stream order and leave its first 4096 bytes zero; the buffer
 * must stay allocated while registered. Plays the part of the scratch
 * allocator the reference installs for its Triton kernels
 * (fused_forward.py:68-74, triton.set_allocator). */
int swiglu_b200_set_stream_workspace(void* workspace, size_t bytes, void* stream);

/* One launch: preact [M, 2H] = x [M, K] . W1^T and h [M, H] = left * silu(gate).
 * h may be NULL (preact only); preact may be NULL (h only: the no-save
 * inference forward, the external `fused_swiglu_wide_packed` that
 * bench_packed_vs_cublas.py:25-30,72 measures).
 *   w_form = T, layout = STD:       fused_matmul_swiglu_save_preact   fused_forward.py:188-256
 *   w_form = T, layout = PACKED128: fused_swiglu_save_preact_packed    fused_forward_packed.py:186-216
 *                                   (and fused_forward_packed_canon.py:103-134)
 *   w_form = ROWS, layout = STD:    `x @ W1.t()` + `_swiglu_forward_logic` swiglu_recompute.py:61,64
 * h_from_rounded_preact = 1 computes h from the stored (rounded) preact, as the
 * recompute Function does (swiglu_recompute.py:64); 0 computes it from the f32
 * accumulator, as the fused Triton kernels do (fused_forward.py:177).
 * group_size_m: L2 swizzle group of the tile order (fused_forward.py:192). */
int swiglu_b200_fused_matmul_swiglu_save_preact(const void* x, const void* w, void* preact, void* h, int64_t M,
                                                int64_t K, int64_t H, int dtype, int w_form, int layout,
                                                int h_from_rounded_preact, int group_size_m, void* stream);

/* C [M, N] = op(A) . op(B), f32 accumulation; out_dtype may be F32 for a bf16 GEMM.
 *   a_layout 0: A stored [M, K];  1: A stored [K, M] (op(A) = stored^T)
 *   b_layout 0: B stored [K, N];  1: B stored [N, K] (op(B) = stored^T)
 * Replaces the torch.matmul calls of the path: y = h @ W2.t() (swiglu_recompute.py:65),
 * grad_W1 = grad_preact.t() @ x (:76), grad_x = grad_preact @ W1 (:77), and their
 * w1t/packed forms (fused_forward.py:272,282-283; fused_forward_packed.py:301,314-315). */
int swiglu_b200_matmul(const void* a, const void* b, void* c, int64_t M, int64_t N, int64_t K, int a_layout,
                       int b_layout, int dtype, int out_dtype, int group_size_m, void* stream);

/* swiglu_b200_matmul with a preferred output-tile width for the 2-SM kernel:
 * tile_n = 256 (256 x 256 tiles, accumulator double-buffered in TMEM), 512
 * (256 x 512 tiles: a quarter fewer operand bytes per FLOP, epilogue between
 * main loops; used for the backward's long-K GEMMs dW1 = grad_preact^T . x
 * and dx = grad_preact . W1, swiglu_recompute.py:76-77) or 0 (by size: 512
 * once the 256 x 512 tiles make 8 waves of CTA pairs, else 256; this is what
 * swiglu_b200_matmul does). A path forced with swiglu_b200_set_gemm_path takes
 * precedence. */
int swiglu_b200_matmul_tiled(const void* a, const void* b, void* c, int64_t M, int64_t N, int64_t K, int a_layout,
                             int b_layout, int dtype, int out_dtype, int group_size_m, int tile_n, void* stream);

/* Tensor-parallel reduce-scatter fused into a GEMM (used for the partial y
 * and grad_x of the tensor-parallel block). The f32 result D [M, N] =
 * op(A) . op(B) is not stored locally: row r goes to rank o = r / rows_per_rank,
 * into peer_bufs[o] (a device pointer valid on this GPU, usually another GPU's
 * memory mapped over NVLink) at row rank * rows_per_rank + r % rows_per_rank of
 * a [world * rows_per_rank, N] f32 receive buffer. peer_bufs is a host array of
 * `world` pointers; M == world * rows_per_rank; bf16 operands; world <= 8.
 * Replaces the NCCL reduce-scatter after `h @ W2.t()` / `grad_preact @ W1` of a
 * tensor-parallel block (the reference is single-GPU; the math per rank is
 * swiglu_recompute.py:65,77). */
int swiglu_b200_matmul_scatter_rows(const void* a, const void* b, int64_t M, int64_t N, int64_t K, int a_layout,
                                    int b_layout, int dtype, void* const* peer_bufs, int world, int rank,
                                    int64_t rows_per_rank, void* stream);

/* After the preceding work on `stream`: publishes `epoch` into
 * peer_flags[o][rank] for every owner o (peer_flags: host array of `world`
 * device pointers to each rank's flag array of `world` uint32). */
int swiglu_b200_tp_signal(uint32_t* const* peer_flags, int world, int rank, uint32_t epoch, void* stream);

/* Owner side: waits (bounded; timeout sets a device status bit) until
 * flags[s] == epoch for every source s, then out [rows, N] = sum over
 * s = 0..world-1 of recv[s] [rows, N] in that order (f32), stored as out_dtype. */
int swiglu_b200_tp_reduce_rows(const float* recv, const uint32_t* flags, int world, uint32_t epoch, void* out,
                               int64_t rows, int64_t N, int out_dtype, void* stream);

/* The tensor-parallel GEMM -> reduce pipeline above for a single rank
 * (matmul_scatter_rows + tp_signal + tp_reduce_rows with world = 1), for callers
 * that cannot allocate device memory: code embedded in a host application
 * whose own pool owns the whole device and forbids cudaMalloc, or code on a
 * path where cudaMalloc's implicit device synchronisation is not allowed.
 * Computes out [M, N] = op(A) . op(B) (bf16 operands, f32 accumulation,
 * out_dtype result) through the library's static device scratch instead of a
 * caller-provided receive buffer; no device memory is allocated.
 * Limit: M * N <= 4,194,304 (16 MiB of f32 scratch, held on every GPU that
 * loads the library until the process exits); larger sizes are rejected with
 * SWIGLU_ERR_INVALID_ARGUMENT. All calls share that scratch: calls that
 * overlap on the GPU (e.g. on different streams) race. The first call on a
 * device resolves the scratch address for that device; make that first call
 * before any stream capture. No counterpart in the reference. */
int swiglu_b200_matmul_reduce_rows_noalloc(const void* a, const void* b, void* out, int64_t M, int64_t N,
                                           int64_t K, int a_layout, int b_layout, int out_dtype, void* stream);

/* dW2 [Dout, H] = grad_y^T . h with h = left * silu(gate) recomputed from preact
 * inside the GEMM's operand prologue (no [M, H] buffer).
 * Replaces `h = _swiglu_forward_logic(preact); grad_W2 = grad_y.t() @ h`
 * (swiglu_recompute.py:71-73; packed: fused_forward_packed.py:310-311). */
int swiglu_b200_bwd_dw2(const void* grad_y, const void* preact, void* dw2, int64_t M, int64_t H, int64_t Dout,
                        int dtype, int layout, void* stream);

/* grad_h = grad_y [M, Dout] . W2 [Dout, H], never stored: the GEMM epilogue turns
 * each tile into grad_left / grad_gate and overwrites preact with grad_preact.
 * Replaces `grad_h = grad_y @ W2; grad_preact = _swiglu_backward_logic(preact, grad_h)`
 * (swiglu_recompute.py:74-75; packed: fused_forward_packed.py:312-313). */
int swiglu_b200_bwd_grad_preact_inplace(const void* grad_y, const void* w2, void* preact, int64_t M, int64_t H,
                                        int64_t Dout, int dtype, int layout, void* stream);

/* As swiglu_b200_bwd_grad_preact_inplace, and the same epilogue also writes
 * h [M, H] = left * silu(gate) of the preact values it replaces (the forward's
 * sigmoid; the dW2 prologue's h uses a tanh-based sigmoid within 3.5e-6 of
 * it, so the two dW2 forms agree to bf16 rounding). dW2 then is a plain GEMM,
 * swiglu_b200_matmul(grad_y, h, dW2, Dout, H, M, a_layout 1, b_layout 0),
 * with no exp/reciprocal on its tensor-core path; the cost is the transient
 * [M, H] buffer, the h the reference itself materialises in backward
 * (swiglu_recompute.py:71). Replaces swiglu_recompute.py:71,74-75 (packed:
 * fused_forward_packed.py:310,312-313). */
int swiglu_b200_bwd_grad_preact_inplace_emit_h(const void* grad_y, const void* w2, void* preact, void* h, int64_t M,
                                               int64_t H, int64_t Dout, int dtype, int layout, void* stream);

/* h [M, H] = left * silu(gate) from preact [M, 2H].
 * _swiglu_forward_logic (swiglu_recompute.py:26-30); packed: _h_from_packed_preact
 * (fused_forward_packed.py:281-286). H % 8 == 0. */
int swiglu_b200_forward_logic(const void* preact, void* h, int64_t M, int64_t H, int dtype, int layout,
                              void* stream);

/* grad_preact [M, 2H] from preact [M, 2H] and grad_h [M, H] (grad_preact may alias preact).
 * _swiglu_backward_logic (swiglu_recompute.py:33-49); packed: swiglu_packed_grad_de_from_preact
 * (fused_forward_packed.py:262-277). H % 8 == 0. */
int swiglu_b200_backward_logic(const void* preact, const void* grad_h, void* grad_preact, int64_t M, int64_t H,
                               int dtype, int layout, void* stream);

/* Chunk-interleave a [K, 2*N_half] weight ([left | gate] -> packed), or undo it (unpack = 1).
 * pack_swiglu_weight_chunked_torch / unpack_swiglu_weight_chunked_torch
 * (fused_forward_packed.py:77-107). src and dst must not alias. */
int swiglu_b200_pack_weight_chunked(const void* src, void* dst, int64_t K, int64_t N_half, int64_t block_n_half,
                                    int dtype, int unpack, void* stream);

/* e4m3 (FP8) operand path. No counterpart in the reference, which computes
 * in bf16/fp32 only: the same GEMMs with 8-bit operands on the tensor core's
 * f8f6f4 kind, for the forward of a block whose inputs tolerate e4m3
 * rounding. Operands are row-scaled: row r of an [R, C] matrix is stored as
 * q[r, :] = e4m3(v[r, :] * 448 / amax_r) with the f32 dequantisation factor
 * s_r = amax_r / 448 (1 for an all-zero row); products are accumulated in
 * f32 and scaled by s_a[row] * s_b[col] in the epilogue.
 *
 * Quantises the bf16 matrix src [rows, cols] (cols % 8 == 0) into e4m3 bytes
 * dst [rows, cols] and row_scale [rows]. */
int swiglu_b200_quantize_rows_e4m3(const void* src, void* dst, float* row_scale, int64_t rows, int64_t cols,
                                   int dtype, void* stream);

/* GEMM1 + SwiGLU with e4m3 operands: preact [M, 2H] (bf16, may be NULL) and
 * h [M, H] (bf16, may be NULL) from xq [M, K] (row scales x_scale [M]) and
 * w1q [2H, K] (rows in `layout` order: [left | gate] or the 128-chunk
 * interleave; row scales w1_scale [2H]). The bf16 form of the same step is
 * swiglu_b200_fused_matmul_swiglu_save_preact (fused_forward.py:188-256,
 * swiglu_recompute.py:61,64). K % 16 == 0, H % 32 == 0. */
int swiglu_b200_fused_matmul_swiglu_e4m3(const void* xq, const float* x_scale, const void* w1q, const float* w1_scale,
                                         void* preact, void* h, int64_t M, int64_t K, int64_t H, int layout,
                                         int h_from_rounded_preact, int group_size_m, void* stream);

/* C [M, N] = (A . B^T) scaled: aq [M, K] with a_scale [M], bq [N, K] with
 * b_scale [N], both e4m3 K-major; C in out_dtype. The e4m3 form of
 * y = h . W2^T (swiglu_recompute.py:65). K % 16 == 0, N % 8 == 0. */
int swiglu_b200_matmul_e4m3(const void* aq, const float* a_scale, const void* bq, const float* b_scale, void* c,
                            int64_t M, int64_t N, int64_t K, int out_dtype, int group_size_m, void* stream);

/* Whole forward of one MLP block: preact (saved for backward), h (caller's
 * transient workspace [M, H]) and y [M, Dout].
 * SwiGLUMemoryOptimizedFunction.forward (swiglu_recompute.py:59-66),
 * SwiGLUFusedForwardFunction.forward (fused_forward.py:265-273),
 * SwiGLUPackedFusedFunction.forward (fused_forward_packed.py:294-302). */
int swiglu_b200_mlp_forward(const void* x, const void* w1, const void* w2, void* preact, void* h_workspace,
                            void* y, int64_t M, int64_t D, int64_t H, int64_t Dout, int dtype, int w_form,
                            int layout, int h_from_rounded_preact, void* stream);

/* Whole backward of one MLP block. preact is consumed: on return it holds
 * grad_preact. dw1 has the form of w1 (ROWS: [2H, D]; T: [D, 2H] in `layout`).
 * SwiGLUMemoryOptimizedFunction.backward (swiglu_recompute.py:68-78),
 * SwiGLUFusedForwardFunction.backward (fused_forward.py:276-284),
 * SwiGLUPackedFusedFunction.backward (fused_forward_packed.py:305-316). */
int swiglu_b200_mlp_backward(const void* x, const void* w1, const void* w2, void* preact, const void* grad_y,
                             void* dx, void* dw1, void* dw2, int64_t M, int64_t D, int64_t H, int64_t Dout,
                             int dtype, int w_form, int layout, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* SWIGLU_B200_H */
