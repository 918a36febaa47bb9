"""Canonical-form packed fused SwiGLU forward (B200 build).

Drop-in for the reference module of the same name
(fused_forward_packed_canon.py). The reference variant defers the tile_id of
the epilogue stores so the Triton compiler overlaps tile T's epilogue with
tile T+1's K-loop (fused_forward_packed_canon.py:66-100). The native kernel
does that overlap structurally: the accumulator is double-buffered in TMEM and
the epilogue warps drain tile T while the MMA warp runs tile T+1. The
canonical entry points therefore launch the same kernel as the packed ones and
return identical results.
"""

from __future__ import annotations

import torch
import torch.nn as nn

from fused_forward_packed import (  # noqa: F401
    BLOCK_SIZE_K,
    BLOCK_SIZE_M,
    BLOCK_SIZE_N_HALF,
    GROUP_SIZE_M,
    NUM_STAGES,
    NUM_WARPS,
    WARP_SPECIALIZE,
    _compute_pid,
    _ensure_allocator,
    _h_from_packed_preact,
    _num_sms,
    fused_swiglu_save_preact_packed,
    pack_swiglu_linear_weight,
    swiglu_packed_grad_de_from_preact,
    unpack_swiglu_linear_weight,
)
from swiglu_b200.ops import LAYOUT_PACKED128, W1_T
from swiglu_b200.library import kernels
from swiglu_recompute import _recompute_backward


def fused_swiglu_save_preact_packed_canon(x, packed_weight):
    """One launch (canonical-form): (h [M,H], preact_packed [M,2H])."""
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


class SwiGLUPackedFusedFunctionCanon(torch.autograd.Function):
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
        h, preact = fused_swiglu_save_preact_packed_canon(x, packed_weight)
        ctx.save_for_backward(x, packed_weight, w2, preact)
        return K.matmul(h, w2, False, True)

    @staticmethod
    def backward(ctx, grad_y):
        x, packed_weight, w2, preact = ctx.saved_tensors
        return _recompute_backward(ctx, grad_y, x, packed_weight, w2, preact,
                                   w_form=W1_T, layout=LAYOUT_PACKED128)


class SwiGLUMLPPackedFusedCanon(nn.Module):
    """SwiGLU MLP with the canonical-form fused forward."""

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
        return SwiGLUPackedFusedFunctionCanon.apply(x, self.packed_weight, self.w2)
