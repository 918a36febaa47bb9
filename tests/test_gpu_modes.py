"""Inference (no-save) forward and full-checkpoint mode. GPU only.

- With no input requiring a gradient, the Functions run the no-save forward
  (GEMM1 writes h only, nothing is saved); y must equal the training forward's.
- SwiGLUFullCheckpointFunction saves only x and recomputes preact in backward;
  its outputs and gradients must equal SwiGLUMemoryOptimizedFunction's bit for
  bit, it must not save an [M, 2H] tensor, and its peak memory is lower.
- The two dW2 modes of the backward ("prologue", the default: h recomputed
  in the dW2 kernel's operand prologue; "emit_h": h written by the grad_h
  epilogue, dW2 a plain GEMM) give bit-identical y, dx and dW1 and dW2 within the bf16
  bound of each other and of the oracle, for every module.
"""
import pytest
import torch

from swiglu_b200 import ops
import fused_forward as FF
import fused_forward_packed as FP
import swiglu_recompute as SR
from oracle import swiglu_oracle as O

pytestmark = pytest.mark.gpu


def _mods(D, H, Dout, w1, w2):
    rc = SR.SwiGLUMLPCustom(D, H, Dout, dtype=torch.bfloat16)
    fc = SR.SwiGLUMLPFullCheckpoint(D, H, Dout, dtype=torch.bfloat16)
    fu = FF.SwiGLUMLPFused(D, H, Dout, dtype=torch.bfloat16)
    pk = FP.SwiGLUMLPPackedFused(D, H, Dout, dtype=torch.bfloat16)
    with torch.no_grad():
        for m in (rc, fc):
            m.w1.copy_(w1)
        fu.w1t.copy_(w1.t().contiguous())
        pk.packed_weight.copy_(FP.pack_swiglu_linear_weight(w1.contiguous()))
        for m in (rc, fc, fu, pk):
            m.w2.copy_(w2)
    return [m.cuda() for m in (rc, fc, fu, pk)]


def test_inference_forward_equals_training_forward():
    M, D, H, Dout = 384, 256, 512, 192
    x, w1, w2, _ = O.make_inputs(M, D, H, Dout, seed=31, dtype=torch.bfloat16)
    xd = x.cuda()
    for m in _mods(D, H, Dout, w1, w2):
        y_train = m(xd.clone().requires_grad_(True)).detach()
        with torch.no_grad():
            y_inf = m(xd)
        assert torch.equal(y_inf, y_train), type(m).__name__
    h_save, _ = FP.fused_swiglu_save_preact_packed(xd, _mods(D, H, Dout, w1, w2)[3].packed_weight.detach())
    h_nosave = FP.fused_swiglu_packed_no_save(xd, _mods(D, H, Dout, w1, w2)[3].packed_weight.detach())
    assert torch.equal(h_save, h_nosave)


def test_full_checkpoint_is_bitwise_recompute():
    M, D, H, Dout = 512, 384, 640, 256
    x, w1, w2, gy = O.make_inputs(M, D, H, Dout, seed=32, dtype=torch.bfloat16)
    rc, fc, _, _ = _mods(D, H, Dout, w1, w2)
    outs = []
    for m in (rc, fc):
        xd = x.cuda().requires_grad_(True)
        y = m(xd)
        g = torch.autograd.grad(y, [xd, m.w1, m.w2], gy.cuda())
        outs.append([y.detach()] + list(g))
    for a, b in zip(*outs):
        assert torch.equal(a, b)
    xd = x.cuda().requires_grad_(True)
    y = fc(xd)
    shapes = [tuple(t.shape) for t in y.grad_fn.saved_tensors]
    assert (M, 2 * H) not in shapes and (M, D) in shapes


def _peak_mib(model, x0, gout):
    params = list(model.parameters())
    for _ in range(2):
        xi = x0.detach().requires_grad_(True)
        torch.autograd.grad(model(xi), [xi] + params, gout)
    torch.cuda.synchronize()
    torch.cuda.reset_peak_memory_stats()
    base = torch.cuda.memory_allocated()
    xi = x0.detach().requires_grad_(True)
    torch.autograd.grad(model(xi), [xi] + params, gout)
    torch.cuda.synchronize()
    return (torch.cuda.max_memory_allocated() - base) / 2 ** 20


def test_full_checkpoint_stack_uses_less_memory():
    M, D, H, N = 2048, 512, 1536, 4
    x0 = torch.randn(M, D).to(torch.bfloat16).cuda()
    gout = torch.randn(M, D).to(torch.bfloat16).cuda()
    peaks = {}
    for cls in (SR.SwiGLUMLPCustom, SR.SwiGLUMLPFullCheckpoint):
        torch.manual_seed(0)
        model = torch.nn.Sequential(*[cls(D, H, D, dtype=torch.bfloat16) for _ in range(N)]).cuda()
        peaks[cls.__name__] = _peak_mib(model, x0, gout)
        del model
        torch.cuda.empty_cache()
    assert peaks["SwiGLUMLPFullCheckpoint"] < peaks["SwiGLUMLPCustom"], peaks


@pytest.mark.parametrize("M,D,H,Dout", [(512, 384, 640, 256), (1024, 512, 768, 384)])
def test_dw2_modes_agree(M, D, H, Dout):
    x, w1, w2, gy = O.make_inputs(M, D, H, Dout, seed=33, dtype=torch.bfloat16)
    ref = O.mlp_forward_backward(x.float(), w1.float(), w2.float(), gy.float(), bf16=True)
    for m in _mods(D, H, Dout, w1, w2):
        res = {}
        default = ops.dw2_mode()
        assert default == "prologue"          # the north star's backward is the default
        for mode in ops.DW2_MODES:
            ops.set_dw2_mode(mode)
            try:
                xd = x.cuda().requires_grad_(True)
                y = m(xd)
                res[mode] = [y.detach()] + list(torch.autograd.grad(y, [xd] + list(m.parameters()), gy.cuda()))
            finally:
                ops.set_dw2_mode(default)
        a, b = res["emit_h"], res["prologue"]
        name = type(m).__name__
        for i in range(3):                        # y, dx, grad of the first-layer weight
            assert torch.equal(a[i], b[i]), (name, i)
        assert O.rel_max(a[3].cpu(), b[3].cpu().float()) <= 8e-3, name
        assert O.rel_max(a[3].cpu(), ref["dw2"]) <= 8e-3, name
        assert O.rel_max(b[3].cpu(), ref["dw2"]) <= 8e-3, name
