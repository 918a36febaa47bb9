"""Parity of the bench line's own step at its full size.

GPU only. Config 2 of the benchmark (M=11136 D=3584 H=14336 Dout=3584, bf16)
runs exactly as `bench.py` runs it: the same seeded draw, SwiGLUMLPCustom's
forward and one autograd.grad, the default kernel choice (CTA-pair kernels,
256 x 512 tiles for dW1 and dx) and a registered stream-K workspace, so the
GEMMs whose last round is mostly idle (y, dx; dW2 in the prologue mode) split
their tail tiles along K and the last-arriving warp sums the f32 parts.

Checked, in both dW2 modes:
  - y, dx, dW1, dW2 against the reference's own bf16 arithmetic on the same
    GPU (swiglu_recompute.py:58-78 op for op, cuBLAS GEMMs): rel_max <= 7e-3,
    or one bf16 ulp of the largest element where that is more (the floor
    test_gpu_parity.py explains);
  - sampled rows of y and dx (whole rows; every 29th row of the last tile
    group, rows >= 8192, whose last column tiles are the split tails) and
    sampled hidden units of dW1 (rows
    j and H + j) and dW2 (column j; units >= 13312 are the prologue kernel's
    split tail) against the CPU oracle in f64: exact math within 7e-3 (or
    1.25x the reference rounding's own distance from it), the reference's
    rounding points within 1e-2 (the bounds of test_gpu_parity.py);
  - that the split tails ran: the same step without a stream-K workspace
    gives different bits in y or dx (f32 summation order only) and passes the
    same bounds.
"""
import pytest
import torch

import swiglu_recompute as SR
from oracle import swiglu_oracle as O
from swiglu_b200 import ops
from swiglu_b200.synthetic import make_inputs

pytestmark = pytest.mark.gpu

M, D, H, DOUT = 11136, 3584, 14336, 3584
REFGPU_TOL = 7e-3
EXACT_TOL = 7e-3
ORACLE_TOL = 1e-2

ROWS = sorted({0, 1, 127, 128, 255, 256, 5000, 5567, 8191, *range(8192, M, 29), 10239, 10240, M - 1})
UNITS = sorted({0, 1, 31, 32, 127, 128, 255, 256, 7167, 7168, 13311, *range(13312, H, 37), H - 1})


@pytest.fixture(scope="module")
def inputs():
    return make_inputs(M, D, H, DOUT, seed=0, dtype=torch.bfloat16)


def _sampled(x, w1, w2, gy, bf16):
    """y[ROWS], dx[ROWS], dW1[UNITS | H + UNITS], dW2[:, UNITS] in f64 from the
    same bf16 inputs; with bf16, rounded where the reference rounds."""
    rnd = (lambda t: O._bf16(t)) if bf16 else (lambda t: t)
    X, W1, W2, GY = (t.double() for t in (x, w1, w2, gy))
    R, J = torch.tensor(ROWS), torch.tensor(UNITS)
    pre_r = rnd(X[R] @ W1.t())                                      # swiglu_recompute.py:61
    h_r = O.forward_logic(pre_r, O.STD, bf16)                       # :64
    y_r = rnd(h_r @ W2.t())                                         # :65
    gp_r = O.backward_logic(pre_r, rnd(GY[R] @ W2), O.STD, bf16)    # :74-75
    dx_r = rnd(gp_r @ W1)                                           # :77
    cols = torch.cat([J, H + J])
    pre_c = rnd(X @ W1[cols].t())                                   # [M, left_J | gate_J]
    h_c = O.forward_logic(pre_c, O.STD, bf16)                       # :71 recompute
    dw2_c = rnd(GY.t() @ h_c)                                       # :73
    gp_c = O.backward_logic(pre_c, rnd(GY @ W2[:, J]), O.STD, bf16)
    dw1_c = rnd(gp_c.t() @ X)                                       # :76
    return {"y": y_r, "dx": dx_r, "dw1": dw1_c, "dw2": dw2_c}


@pytest.fixture(scope="module")
def sampled_refs(inputs):
    return _sampled(*inputs, bf16=False), _sampled(*inputs, bf16=True)


@pytest.fixture(scope="module")
def reference_gpu(inputs):
    x, w1, w2, gy = inputs
    return {k: v.float().cpu() for k, v in
            O.reference_path_bf16(x.cuda(), w1.cuda(), w2.cuda(), gy.cuda()).items()}


def _bench_step(inputs):
    x, w1, w2, gy = inputs
    m = SR.SwiGLUMLPCustom(D, H, DOUT, dtype=torch.bfloat16).cuda()
    with torch.no_grad():
        m.w1.copy_(w1)
        m.w2.copy_(w2)
    xd = x.cuda().requires_grad_(True)
    y = m(xd)
    gx, gw1, gw2 = torch.autograd.grad(y, [xd, m.w1, m.w2], gy.cuda())
    torch.cuda.synchronize()
    assert ops.device_status(0) == 0
    return {"y": y.detach().float().cpu(), "dx": gx.float().cpu(), "dw1": gw1.float().cpu(),
            "dw2": gw2.float().cpu()}


def _slice(out):
    R, J = torch.tensor(ROWS), torch.tensor(UNITS)
    return {"y": out["y"][R], "dx": out["dx"][R], "dw1": out["dw1"][torch.cat([J, H + J])],
            "dw2": out["dw2"][:, J]}


def _check(out, reference_gpu, sampled_refs):
    exact, rounded = sampled_refs
    got = _slice(out)
    for k in ("y", "dx", "dw1", "dw2"):
        e_rg = O.rel_max(out[k], reference_gpu[k])
        bound_rg = max(REFGPU_TOL, O.bf16_resolution(reference_gpu[k]))   # as in test_gpu_parity
        assert e_rg <= bound_rg, (k, "refgpu", e_rg, bound_rg)
        e_gt = O.rel_max(got[k].double(), exact[k])
        bound = max(EXACT_TOL, 1.25 * O.rel_max(rounded[k], exact[k]))
        assert e_gt <= bound, (k, "exact f64 sample", e_gt, bound)
        e_or = O.rel_max(got[k].double(), rounded[k])
        assert e_or <= ORACLE_TOL, (k, "oracle f64 sample", e_or)


@pytest.mark.parametrize("mode", ops.DW2_MODES)
def test_config2_bench_step(inputs, reference_gpu, sampled_refs, mode):
    prev = ops.dw2_mode()
    ops.set_dw2_mode(mode)
    try:
        ops.set_stream_k(True)
        split = _bench_step(inputs)
        dev = torch.cuda.current_device()
        assert (dev, torch.cuda.current_stream().cuda_stream) in ops._workspaces
        _check(split, reference_gpu, sampled_refs)
        ops.set_stream_k(False)
        whole = _bench_step(inputs)
        _check(whole, reference_gpu, sampled_refs)
        assert not (torch.equal(split["y"], whole["y"]) and torch.equal(split["dx"], whole["dx"])), \
            "the stream-K tails did not run"
    finally:
        ops.set_stream_k(True)
        ops.set_dw2_mode(prev)
