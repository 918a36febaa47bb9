"""Fused SwiGLU forward: one kernel that outputs BOTH `preact` and `h` (B200 build).

Drop-in for the reference module of the same name (fused_forward.py): same
symbols, signatures, assertions and return order. The Triton kernel is
replaced by a persistent, warp-specialized tcgen05 kernel (libswiglu_b200.so):
TMA stages x and the two [K, 128] column blocks of Wt (left cols [0, H), gate
cols [H, 2H)) for each output tile, one N=256 MMA accumulates both halves in
TMEM, and the epilogue computes h = left * silu(gate) from the f32
accumulator and stores preact (standard [left | gate] layout) and h.

Weight is stored as ``Wt = W1.t()`` with shape ``[K=D, 2H]`` (left = Wt[:, :H],
gate = Wt[:, H:]); ``preact = x @ Wt``.
"""

from __future__ import annotations

import functools

import torch
import torch.nn as nn

from swiglu_b200.library import kernels
from swiglu_b200.ops import LAYOUT_STD, W1_T

# Reuse this project's own elementwise helpers (fused_forward.py:49 imports them).
from swiglu_recompute import _recompute_backward, _swiglu_backward_logic, _swiglu_forward_logic  # noqa: F401

# -----------------------------------------------------------------------------
# Launch config. Same names as the reference (fused_forward.py:55-65); these are
# the native kernel's tile: 128 rows x (128 left + 128 gate) columns, 64-deep
# K stages; the kernel is always warp-specialized (TMA / MMA / epilogue warps).
# -----------------------------------------------------------------------------
BLOCK_SIZE_M = 128
BLOCK_SIZE_N_HALF = 128
BLOCK_SIZE_K = 64
GROUP_SIZE_M = 16
NUM_WARPS = 6
NUM_STAGES = 4
WARP_SPECIALIZE = True
FLATTEN = True


def _tma_alloc(size: int, alignment: int, stream):
    """Kept for API compatibility. TMA descriptors live in kernel parameters,
    so no device scratch is ever requested."""
    return None


def _ensure_allocator() -> None:
    """No-op: the native kernels need no TMA scratch allocator."""
    return None


@functools.cache
def _num_sms(device_index: int) -> int:
    return torch.cuda.get_device_properties(device_index).multi_processor_count


def _compute_pid(tile_id, num_pid_in_group, num_pid_m, GROUP_SIZE_M_):
    """Grouped tile order used by the native scheduler (fused_forward.py:82-94)."""
    group_id = tile_id // num_pid_in_group
    first_pid_m = group_id * GROUP_SIZE_M_
    group_size_m = min(num_pid_m - first_pid_m, GROUP_SIZE_M_)
    pid_m = first_pid_m + ((tile_id % num_pid_in_group) % group_size_m)
    pid_n = (tile_id % num_pid_in_group) // group_size_m
    return pid_m, pid_n


def fused_matmul_swiglu_save_preact(
    x: torch.Tensor,
    wt: torch.Tensor,
    *,
    group_size_m: int = GROUP_SIZE_M,
    warp_specialize: bool = WARP_SPECIALIZE,
) -> tuple[torch.Tensor, torch.Tensor]:
    """One launch: returns (preact [M, 2H], h [M, H]) for ``preact = x @ wt``.

    ``x`` is [M, K]; ``wt`` is [K, 2H] standard layout (left = wt[:, :H]).
    ``group_size_m`` is the L2-swizzle group of the tile order. ``warp_specialize``
    is accepted for compatibility; the native kernel is always warp-specialized.
    """
    _ensure_allocator()
    assert x.is_cuda and wt.is_cuda
    assert x.is_contiguous() and wt.is_contiguous()

    m, k = x.shape
    k2, n2 = wt.shape
    assert k == k2 and n2 % 2 == 0
    n_half = n2 // 2
    assert m % BLOCK_SIZE_M == 0, f"M={m} must be a multiple of {BLOCK_SIZE_M}"
    assert n_half % BLOCK_SIZE_N_HALF == 0, (
        f"H={n_half} must be a multiple of {BLOCK_SIZE_N_HALF}"
    )
    # h from the f32 accumulator, as the reference kernel does (fused_forward.py:177).
    return kernels().swiglu_fwd(x, wt, W1_T, LAYOUT_STD, False, group_size_m)


# -----------------------------------------------------------------------------
# autograd.Function: fused forward, recompute-h backward (same math as
# SwiGLUMemoryOptimizedFunction, but weight is Wt = W1.t() with shape [K, 2H]).
# -----------------------------------------------------------------------------
class SwiGLUFusedForwardFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, wt, w2):
        if not x.is_contiguous():
            x = x.contiguous()
        if not wt.is_contiguous():
            wt = wt.contiguous()
        w2 = w2.contiguous()
        K = kernels()
        if not any(ctx.needs_input_grad[:3]):                # inference: h only
            h = K.swiglu_fwd_h(x, wt, W1_T, LAYOUT_STD, False)
            return K.matmul(h, w2, False, True)
        preact, h = fused_matmul_swiglu_save_preact(x, wt)   # one kernel
        ctx.save_for_backward(x, wt, w2, preact)             # save preact, NOT h
        y = K.matmul(h, w2, False, True)                     # [M, Dout]
        return y

    @staticmethod
    def backward(ctx, grad_y):
        x, wt, w2, preact = ctx.saved_tensors
        return _recompute_backward(ctx, grad_y, x, wt, w2, preact, w_form=W1_T, layout=LAYOUT_STD)


# -----------------------------------------------------------------------------
# nn.Module wrapper. Weight stored transposed (Wt = W1.t(), shape [D, 2H]).
# -----------------------------------------------------------------------------
class SwiGLUMLPFused(nn.Module):
    """SwiGLU MLP using the fused forward kernel + backward recompute of `h`."""

    def __init__(self, dim, hidden_dim, out_dim=None, dtype=torch.float32):
        super().__init__()
        self.dim = dim
        self.hidden_dim = hidden_dim
        self.out_dim = out_dim if out_dim is not None else dim
        # Wt = W1.t(): [D, 2H]  (left = w1t[:, :H], gate = w1t[:, H:])
        self.w1t = nn.Parameter(torch.empty(dim, 2 * hidden_dim, dtype=dtype))
        self.w2 = nn.Parameter(torch.empty(self.out_dim, hidden_dim, dtype=dtype))
        nn.init.xavier_uniform_(self.w1t)
        nn.init.xavier_uniform_(self.w2)

    def forward(self, x):
        return SwiGLUFusedForwardFunction.apply(x, self.w1t, self.w2)
