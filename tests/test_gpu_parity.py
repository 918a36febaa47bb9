"""End-to-end parity of the drop-in modules.

GPU only. Each reference Function (recompute / fused std / packed / packed
canon) runs fwd+bwd on the B200 through its public module API on seeded
inputs, and every output (y, dx, dW1, dW2) is compared, as rel_max
(max|a-b| / max|b|, bench_swiglu_recompute.py:39-41), with:

  exact   the f32 ground truth of the same (bf16-valued) inputs
          bound: bf16 7e-3, fp32 1e-5
  refgpu  the reference's own bf16 arithmetic run on the same GPU (cuBLAS
          bf16 GEMMs, f32 pointwise): the recompute Function's for the
          recompute variant, h from the f32 accumulator for the fused,
          packed and canon variants (as their Triton forward kernels form
          it); bound bf16 7e-3 for every variant (or one bf16 ulp of the
          largest element, 2^-8 .. 2^-7 of it, where that is more: the
          smallest difference a single rounding flip there makes)
  oracle  the CPU restatement with the reference's rounding points
          bound: bf16 1e-2, fp32 1e-5

Why the CPU oracle gets 1e-2 in bf16: a bf16 result flips by one ulp (2^-8
of the element) whenever a different f32 summation order lands on the other
side of a rounding boundary, and the flips compound through the
preact -> grad_h -> grad_preact -> dx chain. Measured on a B200 at
M=512 D=1024 H=2816: the reference's own GPU arithmetic differs from the CPU
oracle by 7.35e-3 in dx, exactly as much as this implementation does, while
both are 5.2e-3 from the exact result and 1.8e-3 from each other.
"""
import pytest
import torch

import fused_forward as FF
import fused_forward_packed as FP
import fused_forward_packed_canon as FPC
import swiglu_recompute as SR
from oracle import swiglu_oracle as O
from swiglu_b200 import ops

pytestmark = pytest.mark.gpu

EXACT_TOL = {torch.bfloat16: 7e-3, torch.float32: 1e-5}
ORACLE_TOL = {torch.bfloat16: 1e-2, torch.float32: 1e-5}
REFGPU_TOL = 7e-3
TOL = ORACLE_TOL


def check_all(out, x, w1, w2, gy, dtype, *, h_from_accumulator=False):
    bf = dtype == torch.bfloat16
    ref = O.mlp_forward_backward(x, w1, w2, gy, bf16=bf, h_from_accumulator=h_from_accumulator)
    gt = O.ground_truth(x.float(), w1.float(), w2.float(), gy.float())
    rg = None
    if bf:
        rg = {k: v.float().cpu() for k, v in
              O.reference_path_bf16(x.cuda(), w1.cuda(), w2.cuda(), gy.cuda(),
                                    h_from_accumulator=h_from_accumulator).items()}
    for k in ("y", "dx", "dw1", "dw2"):
        e_gt, e_or = O.rel_max(out[k], gt[k]), O.rel_max(out[k], ref[k])
        # At small shapes the reference's own bf16 arithmetic can already sit
        # above 7e-3 from the exact result (8.2e-3 for y at M=333 D=264 H=200
        # Dout=72); there the bound is "no worse than the reference path".
        bound = max(EXACT_TOL[dtype], 1.25 * O.rel_max(ref[k], gt[k]))
        assert e_gt <= bound, (k, "exact", e_gt, bound)
        assert e_or <= ORACLE_TOL[dtype], (k, "oracle", e_or)
        if rg is not None:
            # 7e-3, or one bf16 ulp of the largest element where that is more:
            # two bf16 results whose f32 sums differ in order alone flip a
            # rounding now and then, and a flip at the largest element is
            # 2^-8 .. 2^-7 of it (measured: 7.35e-3 in dx of the fused
            # variant at M=512 D=1024 H=2816, one flip at an element of 1.06).
            e_rg = O.rel_max(out[k], rg[k])
            bound_rg = max(REFGPU_TOL, O.bf16_resolution(rg[k]))
            assert e_rg <= bound_rg, (k, "refgpu", e_rg, bound_rg)
VARIANTS = ["recompute", "fused", "packed", "canon"]


def _module(variant, D, H, Dout, dtype, w1_rows, w2):
    if variant == "recompute":
        m = SR.SwiGLUMLPCustom(D, H, Dout, dtype=dtype)
        with torch.no_grad():
            m.w1.copy_(w1_rows)
    elif variant == "fused":
        m = FF.SwiGLUMLPFused(D, H, Dout, dtype=dtype)
        with torch.no_grad():
            m.w1t.copy_(w1_rows.t().contiguous())
    else:
        cls = FP.SwiGLUMLPPackedFused if variant == "packed" else FPC.SwiGLUMLPPackedFusedCanon
        m = cls(D, H, Dout, dtype=dtype)
        with torch.no_grad():
            m.packed_weight.copy_(FP.pack_swiglu_linear_weight(w1_rows.contiguous()))
    with torch.no_grad():
        m.w2.copy_(w2)
    return m.cuda()


def _grad_w1_rows(variant, g):
    if variant == "recompute":
        return g
    if variant == "fused":
        return g.t()
    return FP.unpack_swiglu_linear_weight(g.contiguous())


def run_variant(variant, M, D, H, Dout, dtype, seed=0):
    x, w1, w2, gy = O.make_inputs(M, D, H, Dout, seed=seed, dtype=dtype)
    m = _module(variant, D, H, Dout, dtype, w1, w2)
    xd = x.cuda().requires_grad_(True)
    y = m(xd)
    params = list(m.parameters())
    gx, gw1, gw2 = torch.autograd.grad(y, [xd] + params, gy.cuda())
    out = {"y": y.detach().cpu(), "dx": gx.cpu(), "dw1": _grad_w1_rows(variant, gw1).cpu(), "dw2": gw2.cpu()}
    return (x, w1, w2, gy), out


@pytest.mark.parametrize("variant", VARIANTS)
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("M,D,H,Dout", [
    (512, 1024, 2816 // 128 * 128, 1024),   # config-1 family (H rounded to 128 for packed)
    (256, 512, 384, 256),
])
def test_variant_matches_oracle(variant, dtype, M, D, H, Dout):
    (x, w1, w2, gy), out = run_variant(variant, M, D, H, Dout, dtype)
    check_all(out, x, w1, w2, gy, dtype, h_from_accumulator=variant != "recompute")


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_config1_shape_recompute(dtype):
    # Config 1 of the benchmark: M=512 D=1024 H=2816 Dout=1024 (H % 128 != 0,
    # so only the standard-layout recompute Function applies, as in the reference).
    for seed in (0, 1):
        (x, w1, w2, gy), out = run_variant("recompute", 512, 1024, 2816, 1024, dtype, seed=seed)
        check_all(out, x, w1, w2, gy, dtype)


@pytest.mark.parametrize("variant", ["recompute", "packed"])
def test_reference_selftest_shape_bf16(variant):
    # The reference self-test shape (fused_forward.py:320-321): D=3584 H=14336 M=512.
    (x, w1, w2, gy), out = run_variant(variant, 512, 3584, 14336, 3584, torch.bfloat16, seed=0)
    check_all(out, x, w1, w2, gy, torch.bfloat16, h_from_accumulator=variant != "recompute")


def test_ragged_shapes_recompute():
    # M not a multiple of the 128-row tile, H not a multiple of 128, odd Dout.
    for (M, D, H, Dout) in [(40, 24, 136, 16), (333, 264, 200, 72), (1, 64, 8, 8)]:
        for dtype in (torch.bfloat16, torch.float32):
            (x, w1, w2, gy), out = run_variant("recompute", M, D, H, Dout, dtype, seed=M)
            check_all(out, x, w1, w2, gy, dtype)


def test_leading_batch_dims():
    D, H, Dout = 128, 256, 64
    x, w1, w2, gy = O.make_inputs(6 * 32, D, H, Dout, seed=5, dtype=torch.bfloat16)
    m = _module("recompute", D, H, Dout, torch.bfloat16, w1, w2)
    xd = x.view(6, 32, D).cuda().requires_grad_(True)
    y = m(xd)
    assert y.shape == (6, 32, Dout)
    gx, = torch.autograd.grad(y, [xd], gy.view(6, 32, Dout).cuda())
    ref = O.mlp_forward_backward(x, w1, w2, gy, bf16=True)
    assert O.rel_max(y.detach().reshape(-1, Dout).cpu(), ref["y"]) <= 7e-3
    assert O.rel_max(gx.reshape(-1, D).cpu(), ref["dx"]) <= 7e-3


@pytest.mark.parametrize("path", [1, 2])
def test_forced_gemm_path_full_step(path):
    from swiglu_b200 import _lib
    _lib.set_gemm_path(path)
    try:
        (x, w1, w2, gy), out = run_variant("recompute", 600, 512, 640, 384, torch.bfloat16, seed=4)
        check_all(out, x, w1, w2, gy, torch.bfloat16)
    finally:
        _lib.set_gemm_path(0)


def test_bitwise_deterministic():
    outs = [run_variant("recompute", 384, 512, 640, 256, torch.bfloat16, seed=9)[1] for _ in range(2)]
    for k in ("y", "dx", "dw1", "dw2"):
        assert torch.equal(outs[0][k], outs[1][k]), k


def test_second_backward_raises():
    D, H, Dout = 64, 128, 64
    x, w1, w2, gy = O.make_inputs(128, D, H, Dout, dtype=torch.bfloat16)
    m = _module("recompute", D, H, Dout, torch.bfloat16, w1, w2)
    xd = x.cuda().requires_grad_(True)
    y = m(xd)
    torch.autograd.grad(y, [xd], gy.cuda(), retain_graph=True)
    with pytest.raises(RuntimeError):
        torch.autograd.grad(y, [xd], gy.cuda())


def test_h_is_not_saved():
    D, H, Dout, M = 192, 640, 128, 384
    x, w1, w2, gy = O.make_inputs(M, D, H, Dout, dtype=torch.bfloat16)
    m = _module("recompute", D, H, Dout, torch.bfloat16, w1, w2)
    xd = x.cuda().requires_grad_(True)
    y = m(xd)
    saved = y.grad_fn.saved_tensors
    shapes = sorted(tuple(t.shape) for t in saved)
    assert (M, H) not in shapes
    assert (M, 2 * H) in shapes


def test_reference_helpers_and_entry_points():
    M, D, H = 256, 256, 256
    x, w1, w2, gy = O.make_inputs(M, D, H, 64, dtype=torch.bfloat16)
    wt = w1.t().contiguous()
    preact, h = FF.fused_matmul_swiglu_save_preact(x.cuda(), wt.cuda())
    ref_pre = O._bf16(x.float() @ wt.float())
    assert O.rel_max(preact.cpu(), ref_pre) <= 7e-3
    assert O.rel_max(SR._swiglu_forward_logic(preact).cpu(), O.forward_logic(preact.cpu(), bf16=True)) <= 7e-3
    gh = torch.randn(M, H, dtype=torch.bfloat16)
    gp = SR._swiglu_backward_logic(preact, gh.cuda())
    assert O.rel_max(gp.cpu(), O.backward_logic(preact.cpu(), gh, bf16=True)) <= 7e-3
    pw = FP.pack_swiglu_linear_weight(w1.cuda())
    hp, pp = FP.fused_swiglu_save_preact_packed(x.cuda(), pw)
    hc, pc = FPC.fused_swiglu_save_preact_packed_canon(x.cuda(), pw)
    assert torch.equal(hp, hc) and torch.equal(pp, pc)
    assert O.rel_max(hp.cpu(), h.cpu()) <= 7e-3
    gde = FP.swiglu_packed_grad_de_from_preact(pp, gh.cuda())
    assert O.rel_max(gde.cpu(), O.backward_logic(pp.cpu(), gh, O.PACKED, bf16=True)) <= 7e-3
    hpk = FP._h_from_packed_preact(pp, M, H // 128, 128)
    assert O.rel_max(hpk.cpu(), O.forward_logic(pp.cpu(), O.PACKED, bf16=True)) <= 7e-3
    with pytest.raises(AssertionError):
        FF.fused_matmul_swiglu_save_preact(x[:100].cuda(), wt.cuda())      # M % 128
    assert ops.device_status(0) == 0
