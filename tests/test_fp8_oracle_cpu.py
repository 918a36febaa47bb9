"""The oracle's e4m3 restatement on the CPU (no GPU): the properties the
kernels are held to by tests/test_gpu_fp8.py, checked on the checker itself,
and the C-ABI argument checks of the e4m3 entry points."""
import ctypes

import torch

from oracle import swiglu_oracle as O
from swiglu_b200 import _lib


def test_quantize_rows_round_trip_and_edges():
    g = torch.Generator().manual_seed(0)
    t = (torch.randn(64, 200, generator=g) * torch.logspace(-6, 6, 64)[:, None]).to(torch.bfloat16)
    t[3] = 0
    q, s = O.quantize_rows_e4m3(t)
    assert q.dtype == torch.float8_e4m3fn and s.dtype == torch.float32
    assert s[3] == 1 and torch.all(q[3].float() == 0)
    v = t.double()
    d = O.dequantize_rows(q, s)
    # e4m3: 3 mantissa bits (half an ulp is 2^-4 of the value) down to the
    # smallest normal 2^-6; below it, subnormal steps of 2^-9 (half: 2^-10).
    bound = torch.maximum(v.abs() * 2 ** -4, s.double()[:, None] * 2 ** -10) * (1 + 1e-6)
    assert torch.all((d - v).abs() <= bound)
    # every row's largest element lands on 448 exactly
    nz = v.abs().amax(1) > 0
    assert torch.all(q.float().abs().amax(1)[nz] == 448.0)


def test_fp8_forward_is_close_to_the_exact_block():
    x, w1, w2, _ = O.make_inputs(64, 128, 128, 64, seed=1, dtype=torch.bfloat16)
    r = O.fp8_forward(x, w1, w2)
    exact = O.mlp_forward_backward(x.double(), w1.double(), w2.double(), torch.zeros(64, 64, dtype=torch.float64))
    assert O.rel_max(r["y"], exact["y"]) < 0.1


def test_e4m3_entry_points_reject_bad_arguments():
    lib = _lib.load()
    p = ctypes.c_void_p(16)
    # quantize: bf16 only, cols % 8
    assert lib.swiglu_b200_quantize_rows_e4m3(p, p, p, 4, 16, _lib.F32, None) == 1
    assert lib.swiglu_b200_quantize_rows_e4m3(p, p, p, 4, 12, _lib.BF16, None) == 1
    # GEMM1 + SwiGLU: K % 16, H % 32, null scale
    f = lib.swiglu_b200_fused_matmul_swiglu_e4m3
    assert f(p, p, p, p, p, p, 128, 24, 64, 0, 1, 16, None) == 1
    assert b"multiple of 16" in lib.swiglu_b200_last_error_message()
    assert f(p, p, p, p, p, p, 128, 32, 48, 0, 1, 16, None) == 1
    assert b"multiple of 32" in lib.swiglu_b200_last_error_message()
    assert f(p, None, p, p, p, p, 128, 32, 64, 0, 1, 16, None) == 1
    assert b"null" in lib.swiglu_b200_last_error_message()
    # matmul: K % 16, N % 8
    m = lib.swiglu_b200_matmul_e4m3
    assert m(p, p, p, p, p, 8, 8, 24, _lib.BF16, 16, None) == 1
    assert m(p, p, p, p, p, 8, 12, 32, _lib.BF16, 16, None) == 1
