"""The e4m3 (FP8) operand path against its CPU restatement.

GPU only. The reference has no FP8 path, so parity is stated against the
oracle's restatement of the library's own definitions (oracle
quantize_rows_e4m3 / fp8_forward): the per-row quantisation must agree bit
for bit (same IEEE f32 divisions, round to nearest even), and the GEMMs,
computed from the same e4m3 operands, must agree with the f64 product of the
dequantised operands to the bf16 rounding of their outputs (rel_max <= 8e-3,
as the bf16 kernel tests; f32 outputs 1e-4, the f32 summation of up to 3584
terms). How far e4m3 moves the block from its bf16 result is measured, not
hidden: the forward module's y is also held against the bf16 block's y at
the loose bound e4m3 rounding allows (0.1).
"""
import pytest
import torch

import swiglu_recompute as SR
from oracle import swiglu_oracle as O
from swiglu_b200 import ops

pytestmark = pytest.mark.gpu

DEV = "cuda"
BF16_TOL = 8e-3


def _r(*shape, seed=0, scale=1.0):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(*shape, generator=g) * scale).to(torch.bfloat16)


def test_quantize_rows_bit_exact():
    t = _r(300, 520, seed=1)
    t[7] = 0                                    # an all-zero row: scale 1, q 0
    t[11] *= 1e-30                              # tiny row (e4m3 range after scaling)
    t[12] *= 1e30                               # huge row
    t[13, 5] = 448.0                            # exact saturation point after scaling
    q, s = ops.quantize_rows_e4m3(t.to(DEV))
    rq, rs = O.quantize_rows_e4m3(t)
    assert torch.equal(s.cpu(), rs)
    assert torch.equal(q.cpu().view(torch.uint8), rq.view(torch.uint8))


@pytest.mark.parametrize("layout", [O.STD, O.PACKED])
@pytest.mark.parametrize("rounded", [True, False])
@pytest.mark.parametrize("M,K,H", [(512, 1024, 512), (300, 256, 384), (4096, 512, 256), (256, 208, 256)])
def test_e4m3_swiglu_forward(layout, rounded, M, K, H):
    lay = ops.LAYOUT_STD if layout == O.STD else ops.LAYOUT_PACKED128
    x = _r(M, K, seed=2)
    w1 = _r(2 * H, K, seed=3, scale=K ** -0.5)                   # rows in standard order
    li, gi = O.col_index(H, layout)
    w1_lay = torch.empty_like(w1)
    w1_lay[li], w1_lay[gi] = w1[:H], w1[H:]                       # rows in `layout` order
    xq, xs = ops.quantize_rows_e4m3(x.to(DEV))
    wq, ws = ops.quantize_rows_e4m3(w1_lay.to(DEV))
    preact, h = ops.swiglu_fwd_e4m3(xq, xs, wq, ws, layout=lay, h_from_rounded=rounded)
    ref = O.fp8_forward(x, w1_lay, torch.zeros(8, H), h_from_rounded=rounded, layout=layout)
    assert O.rel_max(preact.float().cpu().double(), ref["preact"]) <= BF16_TOL
    assert O.rel_max(h.float().cpu().double(), ref["h"]) <= BF16_TOL
    # h only (the inference form) gives the same bits
    _, h_only = ops.swiglu_fwd_e4m3(xq, xs, wq, ws, layout=lay, h_from_rounded=rounded, want_preact=False)
    assert torch.equal(h, h_only)
    assert ops.device_status(0) == 0


@pytest.mark.parametrize("out_dtype,tol", [(torch.bfloat16, BF16_TOL), (torch.float32, 1e-4)])
@pytest.mark.parametrize("M,N,K", [(512, 512, 1024), (333, 264, 128), (4096, 1024, 3584), (256, 256, 144)])
def test_e4m3_matmul(out_dtype, tol, M, N, K):
    a = _r(M, K, seed=4)
    b = _r(N, K, seed=5, scale=K ** -0.5)
    aq, as_ = ops.quantize_rows_e4m3(a.to(DEV))
    bq, bs = ops.quantize_rows_e4m3(b.to(DEV))
    c = ops.matmul_e4m3(aq, as_, bq, bs, out_dtype=out_dtype)
    assert c.dtype == out_dtype
    ref = O.dequantize_rows(aq.cpu(), as_.cpu()) @ O.dequantize_rows(bq.cpu(), bs.cpu()).t()
    assert O.rel_max(c.float().cpu().double(), ref) <= tol
    assert ops.device_status(0) == 0


def test_e4m3_forward_module_fwd_bwd():
    M, D, H, Dout = 512, 1024, 1024, 512
    x, w1, w2, gy = O.make_inputs(M, D, H, Dout, seed=6, dtype=torch.bfloat16)
    m8 = SR.SwiGLUMLPFP8Forward(D, H, Dout, dtype=torch.bfloat16).to(DEV)
    mb = SR.SwiGLUMLPCustom(D, H, Dout, dtype=torch.bfloat16).to(DEV)
    with torch.no_grad():
        for m in (m8, mb):
            m.w1.copy_(w1)
            m.w2.copy_(w2)
    xd = x.to(DEV).requires_grad_(True)
    y8 = m8(xd)
    gx, gw1, gw2 = torch.autograd.grad(y8, [xd, m8.w1, m8.w2], gy.to(DEV))
    ref = O.fp8_forward(x, w1, w2)
    assert O.rel_max(y8.detach().float().cpu().double(), ref["y"]) <= 1e-2
    # The backward is the bf16 recompute backward from the e4m3 forward's preact.
    pre = ref["preact"].float()
    h_bwd = O.forward_logic(pre, O.STD, True)
    gh = O._bf16(gy.float() @ w2.float())
    gp = O.backward_logic(pre, gh, O.STD, True)
    for got, want in ((gx, gp @ w1.float()), (gw1, gp.t() @ x.float()), (gw2, gy.float().t() @ h_bwd)):
        assert O.rel_max(got.float().cpu(), O._bf16(want)) <= 1e-2
    # Distance from the bf16 block: the price of e4m3 operands.
    yb = mb(x.to(DEV))
    assert O.rel_max(y8.detach().float().cpu(), yb.detach().float().cpu()) <= 0.1
    assert ops.device_status(0) == 0
