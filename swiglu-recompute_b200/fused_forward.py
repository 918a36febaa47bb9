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


# -----------------------------------------------------------------------------
# Self-test: fused vs ground truth (fp32 + bf16), plus preact/h sanity
# (same checks and tolerances as fused_forward.py:311-371).
# -----------------------------------------------------------------------------
def _selftest():
    import torch.nn.functional as F
    from swiglu_recompute import SwiGLUMLPGroundTruth

    assert torch.cuda.is_available(), "needs a CUDA GPU"
    torch.cuda.set_device(0)
    print(f"torch {torch.__version__} | {torch.cuda.get_device_name(0)}")

    D, H, Dout = 3584, 14336, 3584
    M = 512

    def run(dtype, tol):
        torch.manual_seed(0)
        gt = SwiGLUMLPGroundTruth(D, H, Dout, dtype=dtype).cuda()
        fused = SwiGLUMLPFused(D, H, Dout, dtype=dtype).cuda()
        with torch.no_grad():
            fused.w1t.copy_(gt.w1.t().contiguous())
            fused.w2.copy_(gt.w2)
        x0 = torch.randn(M, D, device="cuda", dtype=dtype)
        xg = x0.detach().clone().requires_grad_(True)
        xf = x0.detach().clone().requires_grad_(True)
        yg = gt(xg)
        yf = fused(xf)
        gout = torch.randn_like(yg)
        gg = torch.autograd.grad(yg, [xg, gt.w1, gt.w2], gout)
        gf = torch.autograd.grad(yf, [xf, fused.w1t, fused.w2], gout)

        def rel(a, b):
            denom = b.float().abs().max().clamp_min(1e-6)
            return ((a.float() - b.float()).abs().max() / denom).item()

        checks = {"out": rel(yf, yg), "grad_x": rel(gf[0], gg[0]),
                  "grad_W1": rel(gf[1].t(), gg[1]), "grad_W2": rel(gf[2], gg[2])}
        ok = all(v <= tol for v in checks.values())
        print(f"  [{dtype}] tol={tol:g}")
        for name, v in checks.items():
            print(f"      {name:<9s} rel_max={v:.3e}  {'OK' if v <= tol else 'FAIL'}")
        print(f"  => {'PASS' if ok else 'FAIL'}")
        return ok

    torch.manual_seed(1)
    wt = torch.randn(D, 2 * H, device="cuda", dtype=torch.float32) * (D ** -0.5)
    x = torch.randn(M, D, device="cuda", dtype=torch.float32) * (D ** -0.5)
    preact, h = fused_matmul_swiglu_save_preact(x, wt)
    ref_preact = x @ wt
    left, gate = ref_preact.chunk(2, dim=-1)
    ref_h = left * F.silu(gate)
    print(f"  [sanity fp32] preact max_abs={(preact - ref_preact).abs().max().item():.3e}  "
          f"h max_abs={(h - ref_h).abs().max().item():.3e}")

    ok32 = run(torch.float32, tol=1e-4)
    okbf = run(torch.bfloat16, tol=2e-2)
    print("ALL PASS" if (ok32 and okbf) else "FAILURES PRESENT")
    return ok32 and okbf


if __name__ == "__main__":
    _selftest()
