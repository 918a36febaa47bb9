"""CPU oracle of the SwiGLU-MLP recompute path. TEST INFRASTRUCTURE ONLY.

Only `tests/`, `__graft_entry__.smoke()` and `bench.py`'s CPU-baseline leg
may import this module; it is the checker the native kernels are compared
against, never part of the product path.

A plain-PyTorch (CPU, fp32) restatement of tongzhou8086/swiglu-recompute's
math, one function per reference function (file:line cited on each). The bf16
mode reproduces the reference's rounding points: every GEMM output is rounded
to bf16 once (cuBLAS, f32 accumulation), every compiled pointwise chain runs in
f32 from bf16 inputs and rounds once on store (Inductor).

Pinned against golden vectors produced by running the reference itself
(tests/golden/make_golden.py -> tests/golden/*.npz, checked by
tests/test_oracle_golden.py).
"""
from __future__ import annotations

import math

import torch

STD, PACKED = "std", "packed"
PACK_CHUNK = 128  # BLOCK_SIZE_N_HALF, fused_forward_packed.py:41


def rel_max(a: torch.Tensor, b: torch.Tensor) -> float:
    """max|a-b| / max|b| (bench_swiglu_recompute.py:39-41)."""
    denom = b.float().abs().max().clamp_min(1e-6)
    return ((a.float() - b.float()).abs().max() / denom).item()


def _wide(t: torch.Tensor) -> torch.Tensor:
    """f32 for the arithmetic, unless the caller works in f64 already."""
    return t if t.dtype == torch.float64 else t.float()


def _bf16(t: torch.Tensor) -> torch.Tensor:
    """Round to bf16 and return in the working precision (f32, or f64)."""
    return t.to(torch.bfloat16).to(torch.float64 if t.dtype == torch.float64 else torch.float32)


def _round(t: torch.Tensor, bf16: bool) -> torch.Tensor:
    return _bf16(t) if bf16 else t


def col_index(H: int, layout: str, block: int = PACK_CHUNK):
    """Column index of left[j] and gate[j] in a [.., 2H] row.

    std: [left | gate] (swiglu_recompute.py:29 `chunk(2)`);
    packed: [left0|gate0|left1|...] in `block` chunks (fused_forward_packed.py:77-92).
    """
    j = torch.arange(H)
    if layout == STD:
        return j, j + H
    assert H % block == 0
    c, off = j // block, j % block
    return c * 2 * block + off, c * 2 * block + block + off


def pack_weight_chunked(weight: torch.Tensor, block: int = PACK_CHUNK) -> torch.Tensor:
    """[K, 2N] standard -> chunk-interleaved (fused_forward_packed.py:77-92)."""
    K, n2 = weight.shape
    li, gi = col_index(n2 // 2, PACKED, block)
    out = torch.empty_like(weight)
    out[:, li] = weight[:, : n2 // 2]
    out[:, gi] = weight[:, n2 // 2:]
    return out


def unpack_weight_chunked(packed: torch.Tensor, block: int = PACK_CHUNK) -> torch.Tensor:
    """Inverse of pack_weight_chunked (fused_forward_packed.py:95-107)."""
    K, n2 = packed.shape
    li, gi = col_index(n2 // 2, PACKED, block)
    return torch.cat([packed[:, li], packed[:, gi]], dim=1)


def forward_logic(preact: torch.Tensor, layout: str = STD, bf16: bool = False) -> torch.Tensor:
    """h = left * silu(gate) (swiglu_recompute.py:26-30; packed gather
    fused_forward_packed.py:281-286). f32 math, one rounding."""
    H = preact.shape[-1] // 2
    li, gi = col_index(H, layout)
    p = _wide(preact)
    left, gate = p[:, li], p[:, gi]
    return _round(left * (gate * torch.sigmoid(gate)), bf16)


def backward_logic(preact: torch.Tensor, grad_h: torch.Tensor, layout: str = STD,
                   bf16: bool = False) -> torch.Tensor:
    """grad_preact via the explicit SiLU derivative (swiglu_recompute.py:33-49;
    packed: fused_forward_packed.py:247-259)."""
    H = preact.shape[-1] // 2
    li, gi = col_index(H, layout)
    p = _wide(preact)
    left, gate = p[:, li], p[:, gi]
    g = _wide(grad_h).to(p.dtype)
    sig = torch.sigmoid(gate)
    silu = gate * sig
    dsilu = sig + silu * (1.0 - sig)
    out = torch.empty_like(p)
    out[:, li] = g * silu
    out[:, gi] = g * left * dsilu
    return _round(out, bf16)


def mlp_forward_backward(x, w1_rows, w2, grad_y, *, bf16: bool = False,
                         h_from_accumulator: bool = False, layout: str = STD):
    """One recompute fwd+bwd (SwiGLUMemoryOptimizedFunction, swiglu_recompute.py:58-78).

    w1_rows is W1 [2H, D] with its 2H rows in `layout` order. With
    h_from_accumulator the forward h comes from the unrounded GEMM result, as
    in the fused Triton kernels (fused_forward.py:177,
    fused_forward_packed.py:174-177); the backward is identical in all variants.
    Returns dict(y, dx, dw1, dw2, preact).
    """
    x, w1, w2, gy = (t.float() for t in (x, w1_rows, w2, grad_y))
    acc = x @ w1.t()                                        # :61
    preact = _round(acc, bf16)
    src = acc if h_from_accumulator else preact
    h = forward_logic(src, layout, bf16)                    # :64
    y = _round(h @ w2.t(), bf16)                            # :65
    h_bwd = forward_logic(preact, layout, bf16)             # :71 recompute
    dw2 = _round(gy.t() @ h_bwd, bf16)                      # :73
    grad_h = _round(gy @ w2, bf16)                          # :74
    gp = backward_logic(preact, grad_h, layout, bf16)       # :75
    dw1 = _round(gp.t() @ x, bf16)                          # :76
    dx = _round(gp @ w1, bf16)                              # :77
    return {"y": y, "dx": dx, "dw1": dw1, "dw2": dw2, "preact": preact, "h": h}


def reference_path_bf16(x, w1_rows, w2, grad_y, *, h_from_accumulator: bool = False):
    """The reference's own bf16 arithmetic, op for op: bf16 x bf16 -> bf16
    matmuls (f32 accumulation in the BLAS of whatever device the tensors live
    on) and the pointwise helpers in f32 rounded once. Run on CUDA tensors it
    reproduces what the reference computes on the GPU; the parity tests use it
    there.

    Default: the recompute Function (swiglu_recompute.py:58-78), h from the
    bf16 preact. h_from_accumulator: the fused forward kernels
    (fused_forward.py:165-185, fused_forward_packed.py:167-183), which form h
    from the f32 accumulator of x . W1^T before preact is rounded; their
    backward is the recompute backward (fused_forward.py:277-284,
    fused_forward_packed.py:303-316)."""
    x, w1, w2, gy = (t.to(torch.bfloat16) for t in (x, w1_rows, w2, grad_y))
    if h_from_accumulator:
        acc = x.float() @ w1.float().t()
        preact = acc.to(torch.bfloat16)
        h = forward_logic(acc, STD, True).to(torch.bfloat16)
    else:
        preact = x @ w1.t()
        h = forward_logic(preact.float(), STD, True).to(torch.bfloat16)
    y = h @ w2.t()
    h_bwd = forward_logic(preact.float(), STD, True).to(torch.bfloat16)
    dw2 = gy.t() @ h_bwd
    grad_h = gy @ w2
    gp = backward_logic(preact.float(), grad_h.float(), STD, True).to(torch.bfloat16)
    return {"y": y, "dx": gp @ w1, "dw1": gp.t() @ x, "dw2": dw2}


def bf16_resolution(ref: torch.Tensor) -> float:
    """One bf16 ulp of the largest |element| of `ref`, relative to it: the
    smallest non-zero rel_max that two bf16 results can have when the
    largest element itself differs by a rounding flip (between 2^-8 and 2^-7),
    with 1e-6 of it to spare for rel_max's own f32 evaluation."""
    m = ref.double().abs().max().item()
    if m == 0.0:
        return 0.0
    return 2.0 ** (math.floor(math.log2(m)) - 7) / m * (1.0 + 1e-6)


def bf16_ulps(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """Per-element distance between two bf16-valued tensors in units in the
    last place: how many representable bf16 values lie between them (+0 and
    -0 coincide). Both inputs are cast to bf16 first (exact for bf16 values)."""
    def line(t):
        i = t.to(torch.bfloat16).contiguous().view(torch.int16).to(torch.int32)
        mag = i & 0x7FFF
        return torch.where(i < 0, -mag, mag)
    return (line(a) - line(b)).abs()


def ground_truth(x, w1, w2, grad_y):
    """Autograd through the standard MLP (SwiGLUMLPGroundTruth, swiglu_recompute.py:101-118)."""
    x = x.detach().clone().requires_grad_(True)
    w1 = w1.detach().clone().requires_grad_(True)
    w2 = w2.detach().clone().requires_grad_(True)
    preact = x @ w1.t()
    left, gate = preact.chunk(2, dim=-1)
    y = (left * torch.nn.functional.silu(gate)) @ w2.t()
    dx, dw1, dw2 = torch.autograd.grad(y, [x, w1, w2], grad_y)
    return {"y": y.detach(), "dx": dx, "dw1": dw1, "dw2": dw2}


def make_inputs(M: int, D: int, H: int, Dout: int, seed: int = 0, dtype=torch.float32):
    """Seeded inputs with the distributions of the benchmark configs: x, grad_y ~
    N(0,1); W1, W2 ~ N(0, fan_in^-1/2) (fused_forward.py:359-360). Drawn in
    f32 on the CPU in the order x, W1, W2, grad_y, then cast."""
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(M, D, generator=g)
    w1 = torch.randn(2 * H, D, generator=g) * D ** -0.5
    w2 = torch.randn(Dout, H, generator=g) * H ** -0.5
    gy = torch.randn(M, Dout, generator=g)
    return tuple(t.to(dtype) for t in (x, w1, w2, gy))


# ---------------------------------------------------------------- e4m3 path
# The library's FP8 forward has no counterpart in the reference (which runs
# bf16 / fp32 only). These restate the library's own definitions so its
# kernels can be checked: per-row e4m3 quantisation, then the reference's
# forward math (swiglu_recompute.py:61-65) on the dequantised operands.
def quantize_rows_e4m3(t: torch.Tensor):
    """(q float8_e4m3fn [R, C], scale f32 [R]) of a 2-D tensor: amax_r = max
    |v| over row r, q = e4m3(v * (448 / amax_r)) rounded to nearest even
    (|v * 448 / amax_r| <= 448, so nothing saturates beyond the largest
    finite value), scale_r = amax_r / 448; an all-zero row gets scale 1. Both
    divisions in f32, as the kernel does them."""
    v = t.float()
    amax = v.abs().amax(dim=1)
    nz = amax > 0
    one = torch.ones_like(amax)
    qs = torch.where(nz, torch.full_like(amax, 448.0) / amax, one)
    scale = torch.where(nz, amax / torch.full_like(amax, 448.0), one)
    q = (v * qs[:, None]).to(torch.float8_e4m3fn)
    return q, scale


def dequantize_rows(q: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    """f64 values of a row-scaled e4m3 matrix."""
    return q.double() * scale.double()[:, None]


def fp8_forward(x, w1_rows, w2, *, h_from_rounded: bool = True, layout: str = STD):
    """The e4m3 forward of one block in f64 from bf16 inputs: x, W1 quantised
    per row, preact = deq(x) deq(W1)^T rounded to bf16, h = left * silu(gate)
    (from the rounded preact, or the unrounded product) rounded to bf16, h and
    W2 quantised per row, y = deq(h) deq(W2)^T rounded to bf16. W1's rows are
    in `layout` order. Returns dict(preact, h, y) in f64."""
    xq, xs = quantize_rows_e4m3(x.to(torch.bfloat16))
    wq, ws = quantize_rows_e4m3(w1_rows.to(torch.bfloat16))
    acc = dequantize_rows(xq, xs) @ dequantize_rows(wq, ws).t()
    preact = _bf16(acc)
    h = forward_logic(preact if h_from_rounded else acc, layout, True)
    hq, hs = quantize_rows_e4m3(h.to(torch.bfloat16))
    w2q, w2s = quantize_rows_e4m3(w2.to(torch.bfloat16))
    y = _bf16(dequantize_rows(hq, hs) @ dequantize_rows(w2q, w2s).t())
    return {"preact": preact, "h": h, "y": y}
