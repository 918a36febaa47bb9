"""The no-allocation entry point, swiglu_b200_matmul_reduce_rows_noalloc.

Some callers cannot allocate device memory (an embedding application whose own
pool owns the device and forbids cudaMalloc, or a path where cudaMalloc's
implicit device synchronisation is not allowed). For them the library offers
the single-rank GEMM -> reduce pipeline with its scratch in static device
memory. This test calls it through the C ABI twice in a row, with different
inputs, and checks each result against the same computation through the
existing entry points (caller-allocated receive buffer), within the bf16
tolerance used by the other kernel tests. It also checks that sizes beyond the
static scratch are rejected. GPU only; collected last on purpose.
"""
import ctypes

import pytest
import torch

from oracle import swiglu_oracle as O
from swiglu_b200 import _lib

pytestmark = pytest.mark.gpu

BF16_TOL = 8e-3       # as in test_gpu_kernels.py
SCRATCH_FLOATS = 4 << 20


def _p(t):
    return ctypes.c_void_p(t.data_ptr())


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _code(dtype):
    return _lib.F32 if dtype == torch.float32 else _lib.BF16


def _existing_pipeline(a, b, M, N, K, out_dtype=torch.bfloat16):
    """The same computation through the existing entry points, with a
    caller-allocated receive buffer and flag array (world = 1)."""
    lib = _lib.load()
    recv = torch.empty(M * N, dtype=torch.float32, device="cuda")
    flags = torch.zeros(1, dtype=torch.int32, device="cuda")
    out = torch.empty(M, N, dtype=out_dtype, device="cuda")
    peers = (ctypes.c_void_p * 1)(recv.data_ptr())
    peer_flags = (ctypes.c_void_p * 1)(flags.data_ptr())
    _lib.check(lib.swiglu_b200_matmul_scatter_rows(_p(a), _p(b), M, N, K, 0, 1, _lib.BF16, peers, 1, 0, M,
                                                   _stream()))
    _lib.check(lib.swiglu_b200_tp_signal(peer_flags, 1, 0, 7, _stream()))
    _lib.check(lib.swiglu_b200_tp_reduce_rows(_p(recv), _p(flags), 1, 7, _p(out), M, N, _code(out_dtype),
                                              _stream()))
    return out


def _noalloc(a, b, M, N, K, out_dtype=torch.bfloat16):
    lib = _lib.load()
    out = torch.empty(M, N, dtype=out_dtype, device="cuda")
    _lib.check(lib.swiglu_b200_matmul_reduce_rows_noalloc(_p(a), _p(b), _p(out), M, N, K, 0, 1,
                                                          _code(out_dtype), _stream()))
    return out


def test_noalloc_matches_existing_entry_points_twice_in_a_row():
    torch.cuda.set_device(0)
    g = torch.Generator().manual_seed(21)
    cases = [(640, 1024, 512), (384, 520, 1024)]     # a [M, K], b = W [N, K] (op(B) = W^T)
    for M, N, K in cases:
        a = torch.randn(M, K, generator=g).to(torch.bfloat16).cuda()
        b = (torch.randn(N, K, generator=g) * K ** -0.5).to(torch.bfloat16).cuda()
        got = _noalloc(a, b, M, N, K)
        want = _existing_pipeline(a, b, M, N, K)
        torch.cuda.synchronize()
        assert O.rel_max(got.cpu(), want.cpu()) <= BF16_TOL
        exact = a.float().cpu() @ b.float().cpu().t()
        assert O.rel_max(got.cpu(), exact) <= BF16_TOL
    assert _lib.device_status() == 0


def test_noalloc_at_its_limit_and_with_f32_output():
    """M * N exactly at the scratch size (every scratch float written), then
    an f32 output twice in a row, each against the caller-buffer pipeline
    (bit for bit: same kernels, same summation order) and the exact product."""
    torch.cuda.set_device(0)
    g = torch.Generator().manual_seed(22)
    cases = [(4096, 1024, 256, torch.bfloat16, BF16_TOL),     # M * N == 4,194,304
             (512, 768, 384, torch.float32, 1e-5),
             (4096, 1024, 128, torch.float32, 1e-5)]
    for M, N, K, odt, tol in cases:
        a = torch.randn(M, K, generator=g).to(torch.bfloat16).cuda()
        b = (torch.randn(N, K, generator=g) * K ** -0.5).to(torch.bfloat16).cuda()
        got = _noalloc(a, b, M, N, K, odt)
        want = _existing_pipeline(a, b, M, N, K, odt)
        torch.cuda.synchronize()
        assert got.dtype == odt
        assert torch.equal(got, want)
        exact = a.float().cpu() @ b.float().cpu().t()
        assert O.rel_max(got.float().cpu(), exact) <= tol
    assert M * N == SCRATCH_FLOATS
    assert _lib.device_status() == 0


def test_noalloc_rejects_sizes_beyond_its_scratch():
    lib = _lib.load()
    M, N, K = 4096, 1032, 64           # M * N > 4,194,304
    assert M * N > SCRATCH_FLOATS
    rc = lib.swiglu_b200_matmul_reduce_rows_noalloc(ctypes.c_void_p(16), ctypes.c_void_p(16),
                                                    ctypes.c_void_p(16), M, N, K, 0, 1, _lib.BF16,
                                                    ctypes.c_void_p(0))
    assert rc == 1
    assert b"static scratch" in lib.swiglu_b200_last_error_message()
