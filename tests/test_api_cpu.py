"""The drop-in modules' preconditions without a GPU.

The reference's entry points assert their inputs before any launch
(fused_forward.py:204-214, fused_forward_packed.py:189-195): CUDA tensors,
contiguous, inner dimensions that match. The same AssertionError comes from
this build's modules, in the same order. The product path has no CPU
fallback, so the modules refuse CPU tensors instead of computing on the host.
"""
import pytest
import torch

import fused_forward as FF
import fused_forward_packed as FP
import fused_forward_packed_canon as FC
import swiglu_recompute as SR

M, K, H, DOUT = 256, 128, 256, 64


def _x():
    return torch.randn(M, K, dtype=torch.bfloat16)


def _wt():
    return torch.randn(K, 2 * H, dtype=torch.bfloat16)


@pytest.mark.parametrize("fn", [FF.fused_matmul_swiglu_save_preact, FP.fused_swiglu_save_preact_packed,
                                FP.fused_swiglu_packed_no_save, FC.fused_swiglu_save_preact_packed_canon])
def test_entry_points_assert_cuda_inputs(fn):
    with pytest.raises(AssertionError):
        fn(_x(), _wt())


@pytest.mark.parametrize("cls", [SR.SwiGLUMLPCustom, SR.SwiGLUMLPFullCheckpoint, FF.SwiGLUMLPFused,
                                 FP.SwiGLUMLPPackedFused, FC.SwiGLUMLPPackedFusedCanon])
def test_modules_refuse_cpu_tensors(cls):
    mlp = cls(K, H, DOUT, dtype=torch.bfloat16)
    with pytest.raises((AssertionError, RuntimeError, ValueError)):
        mlp(_x())


def test_modules_keep_the_reference_parameter_shapes():
    """Constructor signature and parameter layout of each module
    (swiglu_recompute.py:84-98, fused_forward.py:290-305,
    fused_forward_packed.py:319-336)."""
    assert SR.SwiGLUMLPCustom(K, H, DOUT).w1.shape == (2 * H, K)
    assert SR.SwiGLUMLPCustom(K, H, DOUT).w2.shape == (DOUT, H)
    assert SR.SwiGLUMLPCustom(K, H).w2.shape == (K, H)
    assert FF.SwiGLUMLPFused(K, H, DOUT).w1t.shape == (K, 2 * H)
    assert FP.SwiGLUMLPPackedFused(K, H, DOUT).packed_weight.shape == (K, 2 * H)
