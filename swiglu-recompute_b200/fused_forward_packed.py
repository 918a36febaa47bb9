"""PACKED fused SwiGLU forward for the recompute scheme (B200 build).

Drop-in for the reference module of the same name (fused_forward_packed.py).
The packed weight layout interleaves left/gate columns in 128-column chunks,
[left0|gate0|left1|gate1|...], so the [K, 256] B tile of one output tile is a
single contiguous TMA region. The forward kernel (tcgen05, warp-specialized,
persistent) emits BOTH outputs from one launch:

    h            [M, H]    the activation, fed into the down-projection
    preact_packed[M, 2H]   raw preactivation, packed [left0|gate0|left1|...],
                           saved for the backward recompute

The backward recomputes h inside the dW2 GEMM's operand prologue and turns
grad_h into packed grad_de inside the grad_h GEMM's epilogue, in place.

Weight is stored packed as ``packed_weight`` of shape ``[K=D, 2H]``.
"""

from __future__ import annotations

import functools

import torch
import torch.nn as nn

from swiglu_b200 import ops
from swiglu_b200.library import kernels
from swiglu_b200.ops import LAYOUT_PACKED128, W1_T
from swiglu_recompute import _recompute_backward

# -----------------------------------------------------------------------------
# Launch config (names as fused_forward_packed.py:40-46; values are the native
# kernel's tile and pipeline).
# -----------------------------------------------------------------------------
BLOCK_SIZE_M = 128
BLOCK_SIZE_N_HALF = 128
BLOCK_SIZE_K = 64
GROUP_SIZE_M = 32
NUM_WARPS = 6
NUM_STAGES = 4
WARP_SPECIALIZE = True


def _tma_alloc(size: int, alignment: int, stream):
    """Kept for API compatibility; no TMA scratch is ever requested."""
    return None


def _ensure_allocator() -> None:
    return None


@functools.cache
def _num_sms(device_index: int) -> int:
    return torch.cuda.get_device_properties(device_index).multi_processor_count


def _compute_pid(tile_id, num_pid_in_group, num_pid_m, GROUP_SIZE_M_):
    """Grouped tile order (fused_forward_packed.py:62-70)."""
    group_id = tile_id // num_pid_in_group
    first_pid_m = group_id * GROUP_SIZE_M_
    group_size_m = min(num_pid_m - first_pid_m, GROUP_SIZE_M_)
    pid_m = first_pid_m + ((tile_id % num_pid_in_group) % group_size_m)
    pid_n = (tile_id % num_pid_in_group) // group_size_m
    return pid_m, pid_n


# -----------------------------------------------------------------------------
# Packing utilities. Packed layout: [left0|gate0|left1|gate1|...] over the
# output dim at block_n_half granularity (fused_forward_packed.py:77-122).
# CUDA tensors are permuted by a native gather kernel; CPU tensors (module
# construction happens on the host) by the equivalent view copies.
# -----------------------------------------------------------------------------
def _pack_host(weight, block_n_half, unpack):
    k, n2 = weight.shape
    n_half = n2 // 2
    chunks = n_half // block_n_half
    out = torch.empty_like(weight)
    if unpack:
        packed = weight.view(k, chunks, 2, block_n_half)
        out[:, :n_half].view(k, chunks, block_n_half).copy_(packed[:, :, 0, :])
        out[:, n_half:].view(k, chunks, block_n_half).copy_(packed[:, :, 1, :])
    else:
        packed = out.view(k, chunks, 2, block_n_half)
        packed[:, :, 0, :].copy_(weight[:, :n_half].view(k, chunks, block_n_half))
        packed[:, :, 1, :].copy_(weight[:, n_half:].view(k, chunks, block_n_half))
    return out


def _pack(weight, block_n_half, unpack):
    if weight.is_cuda and weight.dtype in (torch.float32, torch.bfloat16):
        return ops.pack_chunked(weight, block_n_half, unpack=unpack)
    return _pack_host(weight, block_n_half, unpack)


def pack_swiglu_weight_chunked_torch(weight: torch.Tensor,
                                     block_n_half: int = BLOCK_SIZE_N_HALF) -> torch.Tensor:
    """Pack [K, 2N] (standard [left | gate]) into chunk-interleaved [K, 2N]."""
    assert weight.is_contiguous()
    k, n2 = weight.shape
    assert n2 % 2 == 0
    n_half = n2 // 2
    assert n_half % block_n_half == 0
    return _pack(weight, block_n_half, unpack=False)


def unpack_swiglu_weight_chunked_torch(packed_weight: torch.Tensor,
                                       block_n_half: int = BLOCK_SIZE_N_HALF) -> torch.Tensor:
    """Undo chunk-interleaved packing back to standard [K, 2N]."""
    assert packed_weight.is_contiguous()
    k, n2 = packed_weight.shape
    n_half = n2 // 2
    assert n_half % block_n_half == 0
    return _pack(packed_weight, block_n_half, unpack=True)


def pack_swiglu_linear_weight(linear_weight: torch.Tensor,
                              block_n_half: int = BLOCK_SIZE_N_HALF) -> torch.Tensor:
    """Pack a Linear weight [2N, K] into internal packed [K, 2N]."""
    assert linear_weight.ndim == 2
    return pack_swiglu_weight_chunked_torch(linear_weight.t().contiguous(), block_n_half)


def unpack_swiglu_linear_weight(packed_weight: torch.Tensor,
                                block_n_half: int = BLOCK_SIZE_N_HALF) -> torch.Tensor:
    """Return a Linear weight [2N, K] from internal packed storage."""
    return unpack_swiglu_weight_chunked_torch(
        packed_weight.contiguous(), block_n_half
    ).t().contiguous()


# -----------------------------------------------------------------------------
# Forward: one launch -> (h, preact) (fused_forward_packed.py:186-216)
# -----------------------------------------------------------------------------
def fused_swiglu_save_preact_packed(x, packed_weight):
    """One launch: (h [M,H], preact_packed [M,2H]) for ``x @ packed_weight``."""
    _ensure_allocator()
    assert x.is_cuda and packed_weight.is_cuda
    assert x.is_contiguous() and packed_weight.is_contiguous()
    m, k = x.shape
    k2, n2 = packed_weight.shape
    assert k == k2 and n2 % 2 == 0
    n_half = n2 // 2
    assert m % BLOCK_SIZE_M == 0 and n_half % BLOCK_SIZE_N_HALF == 0
    preact, h = kernels().swiglu_fwd(x, packed_weight, W1_T, LAYOUT_PACKED128, False, GROUP_SIZE_M)
    return h, preact


def fused_swiglu_packed_no_save(x, packed_weight):
    """h [M, H] only: the no-save (inference) packed forward, the kernel the
    reference measures from outside its tree (bench_packed_vs_cublas.py:25-30,72)."""
    assert x.is_cuda and packed_weight.is_cuda
    assert x.is_contiguous() and packed_weight.is_contiguous()
    m, k = x.shape
    k2, n2 = packed_weight.shape
    assert k == k2 and n2 % 2 == 0 and (n2 // 2) % BLOCK_SIZE_N_HALF == 0
    return kernels().swiglu_fwd_h(x, packed_weight, W1_T, LAYOUT_PACKED128, False, GROUP_SIZE_M)


# -----------------------------------------------------------------------------
# Backward pointwise: packed grad_de from packed preact + dy (fresh output)
# (fused_forward_packed.py:262-277)
# -----------------------------------------------------------------------------
def swiglu_packed_grad_de_from_preact(preact, dy):
    """packed grad_de [M,2H] from packed preact [M,2H] + dy [M,H] (fresh out)."""
    _ensure_allocator()
    assert preact.is_contiguous()
    if not dy.is_contiguous():
        dy = dy.contiguous()
    m, n2 = preact.shape
    n_half = n2 // 2
    assert dy.shape == (m, n_half) and n_half % BLOCK_SIZE_N_HALF == 0
    return ops.backward_logic(preact, dy, layout=LAYOUT_PACKED128)


# h recomputed from packed preact (fused_forward_packed.py:281-286).
def _h_from_packed_preact(preact, M, chunks, bnh):
    assert bnh == BLOCK_SIZE_N_HALF, "the native kernels use 128-column chunks"
    assert preact.shape == (M, 2 * chunks * bnh)
    return ops.forward_logic(preact.contiguous(), layout=LAYOUT_PACKED128)


# -----------------------------------------------------------------------------
# autograd.Function: packed fused forward, recompute-from-packed-preact backward.
# -----------------------------------------------------------------------------
class SwiGLUPackedFusedFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, packed_weight, w2):
        if not x.is_contiguous():
            x = x.contiguous()
        if not packed_weight.is_contiguous():
            packed_weight = packed_weight.contiguous()
        w2 = w2.contiguous()
        K = kernels()
        if not any(ctx.needs_input_grad[:3]):                          # inference: h only
            h = K.swiglu_fwd_h(x, packed_weight, W1_T, LAYOUT_PACKED128, False, GROUP_SIZE_M)
            return K.matmul(h, w2, False, True)
        h, preact = fused_swiglu_save_preact_packed(x, packed_weight)  # one kernel
        ctx.save_for_backward(x, packed_weight, w2, preact)            # save preact, NOT h
        y = K.matmul(h, w2, False, True)
        return y

    @staticmethod
    def backward(ctx, grad_y):
        x, packed_weight, w2, preact = ctx.saved_tensors
        return _recompute_backward(ctx, grad_y, x, packed_weight, w2, preact,
                                   w_form=W1_T, layout=LAYOUT_PACKED128)


class SwiGLUMLPPackedFused(nn.Module):
    """SwiGLU MLP using the packed warp-specialized fused forward + recompute bwd."""

    def __init__(self, dim, hidden_dim, out_dim=None, dtype=torch.float32):
        super().__init__()
        self.dim = dim
        self.hidden_dim = hidden_dim
        self.out_dim = out_dim if out_dim is not None else dim
        assert hidden_dim % BLOCK_SIZE_N_HALF == 0
        std = torch.empty(2 * hidden_dim, dim, dtype=dtype)
        nn.init.xavier_uniform_(std)
        self.packed_weight = nn.Parameter(pack_swiglu_linear_weight(std))
        self.w2 = nn.Parameter(torch.empty(self.out_dim, hidden_dim, dtype=dtype))
        nn.init.xavier_uniform_(self.w2)

    def forward(self, x):
        return SwiGLUPackedFusedFunction.apply(x, self.packed_weight, self.w2)
