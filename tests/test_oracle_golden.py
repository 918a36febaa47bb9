"""Pin the CPU oracle against golden vectors recorded from the reference itself
(tests/golden/make_golden.py). CPU only."""
import os

import numpy as np
import pytest
import torch

from oracle import swiglu_oracle as O

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _load(name):
    z = np.load(os.path.join(GOLDEN, name))
    return lambda k: torch.from_numpy(np.array(z[k]))


@pytest.mark.parametrize("name,bf16,tol", [
    ("mlp_f32.npz", False, 1e-6),
    ("mlp_ragged.npz", False, 1e-6),
    # bf16: identical rounding points; residual differences are single-ulp
    # flips from a different f32 summation order inside the CPU matmuls.
    ("mlp_bf16.npz", True, 2e-4),
])
def test_recompute_fwd_bwd_matches_reference(name, bf16, tol):
    t = _load(name)
    r = O.mlp_forward_backward(t("x"), t("w1"), t("w2"), t("gy"), bf16=bf16)
    for k in ("y", "dx", "dw1", "dw2"):
        assert O.rel_max(r[k], t("rc_" + k)) <= tol, k


@pytest.mark.parametrize("name", ["mlp_f32.npz", "mlp_ragged.npz"])
def test_ground_truth_matches_reference(name):
    t = _load(name)
    g = O.ground_truth(t("x"), t("w1"), t("w2"), t("gy"))
    for k in ("y", "dx", "dw1", "dw2"):
        assert O.rel_max(g[k], t("gt_" + k)) <= 1e-6, k


def test_recompute_equals_ground_truth_f32():
    # The reference's published fp32 parity is 4.5e-7 (results_b200.md:19).
    t = _load("mlp_f32.npz")
    for k in ("y", "dx", "dw1", "dw2"):
        assert O.rel_max(t("rc_" + k), t("gt_" + k)) <= 1e-5


def test_pointwise_helpers():
    t = _load("pointwise.npz")
    assert O.rel_max(O.forward_logic(t("preact")), t("h")) <= 1e-6
    assert O.rel_max(O.backward_logic(t("preact"), t("grad_h")), t("grad_preact")) <= 1e-6
    assert O.rel_max(O.forward_logic(t("preact_packed"), O.PACKED), t("h_packed")) <= 1e-6


def test_pack_unpack_exact():
    t = _load("pointwise.npz")
    assert torch.equal(O.pack_weight_chunked(t("w")), t("packed"))
    assert torch.equal(O.pack_weight_chunked(t("w"), 64), t("packed64"))
    assert torch.equal(O.unpack_weight_chunked(t("packed")), t("unpacked"))
    assert torch.equal(O.unpack_weight_chunked(t("packed")), t("w"))
    assert torch.equal(O.pack_weight_chunked(t("lin").t().contiguous()), t("lin_packed"))


def test_packed_column_map_is_a_permutation():
    for H in (128, 256, 1792):
        li, gi = O.col_index(H, O.PACKED)
        allc = torch.cat([li, gi]).sort().values
        assert torch.equal(allc, torch.arange(2 * H))
