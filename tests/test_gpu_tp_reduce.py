"""The owner-side sum of the fused reduce-scatter (swiglu_b200_tp_reduce_rows)
for every rank count it accepts, on one GPU.

The receive buffer [world, rows, N] and the flag array are filled on this
device with every source's epoch already published, so the kernel's bounded
wait passes at once; its output must equal the f32 sum over sources 0..world-1
taken in that order, bit for bit (f32 output), and that sum rounded once
(bf16 output). The multi-GPU tests cover the same kernel behind real peer
pushes. GPU only.
"""
import ctypes

import pytest
import torch

from swiglu_b200 import _lib

pytestmark = pytest.mark.gpu


def _p(t):
    return ctypes.c_void_p(t.data_ptr())


@pytest.mark.parametrize("world", [1, 2, 3, 4, 5, 6, 7, 8])
@pytest.mark.parametrize("out_dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("rows,N", [(1392, 3584), (37, 20)])
def test_owner_sum_in_rank_order(world, out_dtype, rows, N):
    g = torch.Generator(device="cuda").manual_seed(world * 131 + rows)
    recv = torch.randn(world, rows, N, device="cuda", generator=g)
    epoch = 1234 + world
    flags = torch.full((world,), epoch, dtype=torch.int32, device="cuda")
    out = torch.empty(rows, N, dtype=out_dtype, device="cuda")
    _lib.check(_lib.load().swiglu_b200_tp_reduce_rows(
        _p(recv), _p(flags), world, epoch, _p(out), rows, N,
        _lib.F32 if out_dtype == torch.float32 else _lib.BF16,
        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)))
    want = recv[0].clone()
    for s in range(1, world):
        want = want + recv[s]
    assert torch.equal(out, want.to(out_dtype))
    assert _lib.device_status() == 0
