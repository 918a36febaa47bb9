"""The modules under torch.compile. GPU only.

- torch.compile(module, fullgraph=True) traces every module without a graph
  break (the native kernels are registered torch.library ops) and gives the
  same y and gradients as eager, bit for bit: the same kernels run in the same
  order.
- At N=1 the compiled recompute module's peak memory is at most that of the
  compiled standard MLP, the reference's fair baseline
  (bench_fair_compile.py:45), measured as the reference measures it
  (bench_stacked_blocks.py:55-77).
"""
import pytest
import torch

import fused_forward as FF
import fused_forward_packed as FP
import swiglu_recompute as SR
from oracle import swiglu_oracle as O

pytestmark = pytest.mark.gpu

M, D, H, Dout = 1024, 512, 768, 512


def _fwd_bwd(m, x, gy):
    xi = x.detach().clone().requires_grad_(True)
    y = m(xi)
    return [y.detach()] + list(torch.autograd.grad(y, [xi] + list(m.parameters()), gy))


@pytest.mark.parametrize("cls", [SR.SwiGLUMLPCustom, SR.SwiGLUMLPFullCheckpoint, FF.SwiGLUMLPFused,
                                 FP.SwiGLUMLPPackedFused, SR.SwiGLUMLPFP8Forward])
def test_compiled_module_matches_eager(cls):
    torch._dynamo.reset()
    torch.manual_seed(0)
    m = cls(D, H, Dout, dtype=torch.bfloat16).cuda()
    x, _, _, gy = O.make_inputs(M, D, H, Dout, seed=41, dtype=torch.bfloat16)
    x, gy = x.cuda(), gy.cuda()
    eager = _fwd_bwd(m, x, gy)
    compiled = torch.compile(m, fullgraph=True)
    for _ in range(2):                       # second call: the cached graph
        got = _fwd_bwd(compiled, x, gy)
        for a, b in zip(eager, got):
            assert torch.equal(a, b)
    with torch.no_grad():                    # inference graph: h-only forward
        assert torch.equal(compiled(x), eager[0])


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


def test_compiled_memory_at_most_compiled_ground_truth():
    torch._dynamo.reset()
    Mm, Dm, Hm = 4096, 1024, 2816
    x0 = torch.randn(Mm, Dm, dtype=torch.bfloat16, device="cuda")
    gout = torch.randn(Mm, Dm, dtype=torch.bfloat16, device="cuda")
    peaks = {}
    for name, cls in (("gt", SR.SwiGLUMLPGroundTruth), ("recompute", SR.SwiGLUMLPCustom)):
        torch.manual_seed(0)
        m = torch.compile(cls(Dm, Hm, Dm, dtype=torch.bfloat16).cuda())
        peaks[name] = _peak_mib(m, x0, gout)
        del m
        torch.cuda.empty_cache()
    assert peaks["recompute"] <= peaks["gt"] + 1.0, peaks
