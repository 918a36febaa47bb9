"""SwiGLU MLP with backward-pass recomputation of the activation `h` (B200 build).

Drop-in for the reference module of the same name
(tongzhou8086/swiglu-recompute, swiglu_recompute.py): same symbols, same
signatures, same saved state. The forward saves `preact = x @ W1.t()` but not
`h = left * silu(gate)`; the backward recomputes `h` and the SiLU factors from
`preact`.

What runs underneath is libswiglu_b200.so (hand-written sm_100a kernels):
  forward   one tcgen05 GEMM whose epilogue writes preact and h
            (h from the bf16-rounded preact, as swiglu_recompute.py:64 does),
            then y = h @ W2.t() on tcgen05; h is a transient buffer.
  backward  dW2 = grad_y.t() @ h with h recomputed from preact inside the
            dW2 kernel's operand prologue (no [M, H] buffer); then
            grad_h = grad_y @ W2 with the SwiGLU derivative in the epilogue,
            written over preact in place (grad_h never stored, no cat);
            dW1 = grad_preact.t() @ x and dx = grad_preact @ W1 on tcgen05.
            (ops.set_dw2_mode("emit_h") instead has the grad_h epilogue
            write h to a transient buffer for a plain dW2 GEMM.)
fp32 inputs run the same dataflow on fp32 FFMA kernels (correctness mode).

Shapes:  x [M, D]   W1 [2H, D]   W2 [Dout, H]
         preact [M, 2H]   h [M, H]   y [M, Dout]
"""

from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F

from swiglu_b200 import ops
from swiglu_b200.library import kernels
from swiglu_b200.ops import LAYOUT_STD, W1_ROWS


# -----------------------------------------------------------------------------
# Core SwiGLU math helpers (swiglu_recompute.py:26-49): native pointwise kernels
# -----------------------------------------------------------------------------
def _swiglu_forward_logic(preact: torch.Tensor) -> torch.Tensor:
    """h = left * silu(gate), from preact [M, 2H] -> h [M, H]."""
    shape = preact.shape
    p2 = preact.reshape(-1, shape[-1]).contiguous()
    h = ops.forward_logic(p2, layout=LAYOUT_STD)
    return h.reshape(*shape[:-1], shape[-1] // 2)


def _swiglu_backward_logic(preact: torch.Tensor, grad_h: torch.Tensor) -> torch.Tensor:
    """grad_preact [M, 2H] from preact and grad_h [M, H], via the explicit SiLU derivative.

    silu'(z) = sigmoid(z) + silu(z) * (1 - sigmoid(z))
    grad_left = grad_h * silu(gate)
    grad_gate = grad_h * left * silu'(gate)
    """
    shape = preact.shape
    p2 = preact.reshape(-1, shape[-1]).contiguous()
    g2 = grad_h.reshape(-1, grad_h.shape[-1]).contiguous()
    return ops.backward_logic(p2, g2, layout=LAYOUT_STD).reshape(shape)


def _flatten_rows(x: torch.Tensor) -> torch.Tensor:
    x2 = x.reshape(-1, x.shape[-1])
    return x2 if x2.is_contiguous() else x2.contiguous()


def _recompute_backward(ctx, grad_y, x, w1, w2, preact, *, w_form, layout):
    """Shared backward of the three recompute Functions.

    The grad_h GEMM overwrites preact with grad_preact in place; dW1 / dx
    read grad_preact. dW2 is formed by `ops.dw2_mode()`: "prologue" (default)
    runs the dW2 kernel that recomputes h (swiglu_recompute.py:71) in its
    operand prologue first, while preact is intact (no [M, H] buffer);
    "emit_h" has the grad_h epilogue write the recomputed h to a transient
    [M, H] buffer, and dW2 = grad_y^T h is a plain GEMM. When only dW2 is
    needed the prologue kernel always runs. preact is internal to the Function (never
    a graph output), so consuming it is safe; its version counter is bumped so
    that a second backward through the same graph raises instead of reading
    grad_preact as preact.
    """
    eager = not torch.compiler.is_compiling()
    if eager and getattr(ctx, "_preact_consumed", False):
        raise RuntimeError(
            "SwiGLU recompute backward was already run for this graph: the saved preact "
            "was consumed in place (retain_graph / double backward is not supported)")
    K = kernels()
    need_x, need_w1, need_w2 = ctx.needs_input_grad[:3]
    gy = _flatten_rows(grad_y)
    if gy.dtype != preact.dtype:
        gy = gy.to(preact.dtype)
    grad_x = grad_w1 = grad_w2 = None
    emit_h = need_w2 and (need_x or need_w1) and ops.dw2_mode() == "emit_h"
    if need_w2 and not emit_h:
        grad_w2 = K.bwd_dw2(gy, preact, layout)
    if need_x or need_w1:
        h = torch.empty((preact.shape[0], preact.shape[1] // 2), device=preact.device,
                        dtype=preact.dtype) if emit_h else None
        K.bwd_grad_preact_(gy, w2, preact, layout, h)
        gp = preact                                                   # now holds grad_preact
        if eager:
            ctx._preact_consumed = True
            torch.autograd.graph.increment_version(preact)
        if emit_h:
            grad_w2 = K.matmul(gy, h, True, False)                    # [Dout, H] = grad_y^T h
            del h
        # dW1 and dx contract over the long M and 2H axes: 256 x 512 tiles.
        if need_w1:
            if w_form == W1_ROWS:
                grad_w1 = K.matmul(gp, x, True, False, 512)           # [2H, D] = gp^T x
            else:
                grad_w1 = K.matmul(x, gp, True, False, 512)           # [D, 2H] = x^T gp
        if need_x:
            grad_x = K.matmul(gp, w1, False, w_form != W1_ROWS, 512)
    return grad_x, grad_w1, grad_w2


# -----------------------------------------------------------------------------
# Custom autograd.Function: recompute `h` in backward instead of saving it.
# -----------------------------------------------------------------------------
class SwiGLUMemoryOptimizedFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, W1, W2):
        lead = x.shape[:-1]
        x2 = _flatten_rows(x)
        W1c, W2c = W1.contiguous(), W2.contiguous()
        training = any(ctx.needs_input_grad[:3])
        K = kernels()
        # preact [M, 2H] and the transient h [M, H] from one tcgen05 launch;
        # with no gradient needed, the no-save forward writes h only.
        if training:
            preact, h = K.swiglu_fwd(x2, W1c, W1_ROWS, LAYOUT_STD, True)
        else:
            h = K.swiglu_fwd_h(x2, W1c, W1_ROWS, LAYOUT_STD, True)
        y = K.matmul(h, W2c, False, True)                      # [M, Dout] = h W2^T
        del h                                                 # h is NOT retained
        if training:
            ctx.save_for_backward(x2, W1c, W2c, preact)
        ctx.x_shape = x.shape
        return y.reshape(*lead, W2.shape[0])

    @staticmethod
    def backward(ctx, grad_y):
        x, W1, W2, preact = ctx.saved_tensors
        gx, gw1, gw2 = _recompute_backward(ctx, grad_y, x, W1, W2, preact,
                                           w_form=W1_ROWS, layout=LAYOUT_STD)
        if gx is not None:
            gx = gx.reshape(ctx.x_shape)
        return gx, gw1, gw2


class SwiGLUFullCheckpointFunction(torch.autograd.Function):
    """Full-checkpoint variant: saves only x (and the weights), not preact.

    The backward recomputes preact with the GEMM1 kernel (preact only, no h)
    and then runs the same backward as SwiGLUMemoryOptimizedFunction, so its
    results are bit-identical to it. Per block it saves [M, D] instead of
    [M, D] + [M, 2H], for one extra GEMM1 (2*M*D*2H FLOPs) in backward: the
    next memory lever named in the reference's analysis
    (training_memory_forward_vs_backward.md:217-221). No counterpart module
    exists in the reference.
    """

    @staticmethod
    def forward(ctx, x, W1, W2):
        lead = x.shape[:-1]
        x2 = _flatten_rows(x)
        W1c, W2c = W1.contiguous(), W2.contiguous()
        K = kernels()
        h = K.swiglu_fwd_h(x2, W1c, W1_ROWS, LAYOUT_STD, True)
        y = K.matmul(h, W2c, False, True)
        del h
        if any(ctx.needs_input_grad[:3]):
            ctx.save_for_backward(x2, W1c, W2c)
        ctx.x_shape = x.shape
        return y.reshape(*lead, W2.shape[0])

    @staticmethod
    def backward(ctx, grad_y):
        x, W1, W2 = ctx.saved_tensors
        preact = kernels().swiglu_fwd_preact(x, W1, W1_ROWS, LAYOUT_STD)
        gx, gw1, gw2 = _recompute_backward(ctx, grad_y, x, W1, W2, preact, w_form=W1_ROWS, layout=LAYOUT_STD)
        if gx is not None:
            gx = gx.reshape(ctx.x_shape)
        return gx, gw1, gw2


class SwiGLUFP8ForwardFunction(torch.autograd.Function):
    """Forward GEMMs with e4m3 (FP8) operands, backward as the recompute Function.

    x, W1, h and W2 are quantised per row (e4m3, scale amax / 448); GEMM1 +
    SwiGLU and y = h W2^T run on the tensor core's 8-bit kind with f32
    accumulation and the row scales applied in the epilogue. preact (bf16,
    from the dequantised accumulator) is saved as in
    SwiGLUMemoryOptimizedFunction, whose bf16 backward (h recomputed from
    preact) then follows unchanged. No counterpart in the reference (bf16 /
    fp32 only); results differ from the bf16 block by e4m3 rounding of the
    four operands.
    """

    @staticmethod
    def forward(ctx, x, W1, W2):
        lead = x.shape[:-1]
        x2 = _flatten_rows(x)
        W1c, W2c = W1.contiguous(), W2.contiguous()
        training = any(ctx.needs_input_grad[:3])
        K = kernels()
        xq, xs = K.quantize_e4m3(x2)
        w1q, w1s = K.quantize_e4m3(W1c)
        if training:
            preact, h = K.swiglu_fwd_e4m3(xq, xs, w1q, w1s, LAYOUT_STD)
        else:
            h = K.swiglu_fwd_e4m3_h(xq, xs, w1q, w1s, LAYOUT_STD)
        del xq, w1q
        hq, hs = K.quantize_e4m3(h)
        del h
        w2q, w2s = K.quantize_e4m3(W2c)
        y = K.matmul_e4m3(hq, hs, w2q, w2s)
        if training:
            ctx.save_for_backward(x2, W1c, W2c, preact)
        ctx.x_shape = x.shape
        return y.reshape(*lead, W2.shape[0])

    @staticmethod
    def backward(ctx, grad_y):
        x, W1, W2, preact = ctx.saved_tensors
        gx, gw1, gw2 = _recompute_backward(ctx, grad_y, x, W1, W2, preact, w_form=W1_ROWS, layout=LAYOUT_STD)
        if gx is not None:
            gx = gx.reshape(ctx.x_shape)
        return gx, gw1, gw2


# -----------------------------------------------------------------------------
# nn.Module wrapper
# -----------------------------------------------------------------------------
class SwiGLUMLPCustom(nn.Module):
    """SwiGLU MLP (dim -> hidden -> out_dim) using backward recomputation of `h`."""

    def __init__(self, dim, hidden_dim, out_dim=None, dtype=torch.float32):
        super().__init__()
        self.dim = dim
        self.hidden_dim = hidden_dim
        self.out_dim = out_dim if out_dim is not None else dim
        self.w1 = nn.Parameter(torch.empty(2 * hidden_dim, dim, dtype=dtype))
        self.w2 = nn.Parameter(torch.empty(self.out_dim, hidden_dim, dtype=dtype))
        nn.init.xavier_uniform_(self.w1)
        nn.init.xavier_uniform_(self.w2)

    def forward(self, x):
        return SwiGLUMemoryOptimizedFunction.apply(x, self.w1, self.w2)


class SwiGLUMLPFullCheckpoint(SwiGLUMLPCustom):
    """SwiGLUMLPCustom with full checkpointing: saves only x, recomputes preact."""

    def forward(self, x):
        return SwiGLUFullCheckpointFunction.apply(x, self.w1, self.w2)


class SwiGLUMLPFP8Forward(SwiGLUMLPCustom):
    """SwiGLUMLPCustom whose forward GEMMs take e4m3 operands (bf16 weights
    and activations quantised per row on the fly); bf16 recompute backward."""

    def forward(self, x):
        if x.dtype != torch.bfloat16:
            raise TypeError("the e4m3 forward takes bf16 activations")
        return SwiGLUFP8ForwardFunction.apply(x, self.w1, self.w2)


class SwiGLUMLPGroundTruth(nn.Module):
    """Standard SwiGLU MLP relying on PyTorch autograd (saves `h` and `preact`).

    This is the reference's ground-truth model (swiglu_recompute.py:101-118),
    kept as plain PyTorch on purpose: it is the comparison target of the
    parity checks, not part of the native path.
    """

    def __init__(self, dim, hidden_dim, out_dim=None, dtype=torch.float32):
        super().__init__()
        self.dim = dim
        self.hidden_dim = hidden_dim
        self.out_dim = out_dim if out_dim is not None else dim
        self.w1 = nn.Parameter(torch.empty(2 * hidden_dim, dim, dtype=dtype))
        self.w2 = nn.Parameter(torch.empty(self.out_dim, hidden_dim, dtype=dtype))
        nn.init.xavier_uniform_(self.w1)
        nn.init.xavier_uniform_(self.w2)

    def forward(self, x):
        preact = x @ self.w1.t()
        left, gate = preact.chunk(2, dim=-1)
        h = left * F.silu(gate)
        return h @ self.w2.t()
