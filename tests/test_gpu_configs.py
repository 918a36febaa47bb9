"""Parity at the shapes of the benchmark configurations that are not the
bench line. GPU only; bounds and comparisons as in test_gpu_parity.py.

- config 3 (forward-only, packed weight, D=4096 H=14336): the fused packed
  forward's preact and h at M=1024, and the no-save form's h, against the CPU
  oracle with the reference's rounding points;
- config 5 (tensor parallel, D=Dout=8192 H=28672): one rank's share at 8
  ranks (local W1 [2*3584, 8192], local W2 [8192, 3584]) through the full
  recompute fwd+bwd on a 512-row slice, which exercises K=8192 and the
  per-rank N of that configuration;
- config 2 (the bench line) at its full D/H/Dout with a 768-row slice,
  through all four module variants.
"""
import pytest
import torch

import fused_forward_packed as FP
from oracle import swiglu_oracle as O
from swiglu_b200 import ops
from swiglu_b200.ops import LAYOUT_PACKED128, W1_T

from test_gpu_parity import check_all, run_variant

pytestmark = pytest.mark.gpu


def test_config3_packed_forward():
    M, D, H = 1024, 4096, 14336
    x, w1, _, _ = O.make_inputs(M, D, H, 8, seed=3, dtype=torch.bfloat16)
    wp = FP.pack_swiglu_linear_weight(w1.contiguous())            # [D, 2H] packed
    h, preact = FP.fused_swiglu_save_preact_packed(x.cuda(), wp.cuda())
    h_nosave = FP.fused_swiglu_packed_no_save(x.cuda(), wp.cuda())
    acc = x.float() @ w1.float().t()                                # [M, 2H] standard order
    ref_pre = O._round(acc, True)
    ref_h = O.forward_logic(acc, O.STD, True)                       # h from the f32 accumulator
    li, gi = O.col_index(H, O.PACKED)
    pre_std = torch.empty(M, 2 * H)
    got = preact.float().cpu()
    pre_std[:, :H], pre_std[:, H:] = got[:, li], got[:, gi]
    assert O.rel_max(pre_std, ref_pre) <= 7e-3
    assert O.rel_max(h.float().cpu(), ref_h) <= 7e-3
    assert torch.equal(h, h_nosave)


def test_config5_rank_shard_fwd_bwd():
    # 8-way tensor parallel share of M=65536 D=8192 H=28672 Dout=8192: H/8 = 3584.
    (x, w1, w2, gy), out = run_variant("recompute", 512, 8192, 3584, 8192, torch.bfloat16, seed=5)
    check_all(out, x, w1, w2, gy, torch.bfloat16)


@pytest.mark.parametrize("variant", ["recompute", "fused", "packed", "canon"])
def test_config2_dims_row_slice(variant):
    (x, w1, w2, gy), out = run_variant(variant, 768, 3584, 14336, 3584, torch.bfloat16, seed=7)
    check_all(out, x, w1, w2, gy, torch.bfloat16, h_from_accumulator=variant != "recompute")
    assert ops.device_status() == 0
