"""Stream-K tail of the 2-SM kernels. GPU only.

With a stream workspace registered (the default in swiglu_b200.ops), a 2-SM
launch whose tile count leaves the last round of CTA pairs partly idle splits
those tail tiles along K; the parts are summed in part order by whichever
epilogue warp arrives last. The checks, on shapes that take the split:

- the result matches the unsplit kernel (stream-K off) and the fp32 oracle
  within the bf16 bound (8e-3; the two differ only in f32 summation order);
- two runs are bit-identical (the sum order does not depend on timing);
- the split really ran (partials were written) and every arrival counter is
  zero afterwards;
- a stale counter left by an interrupted launch (another epoch's tag) is
  ignored: the result is unchanged and the counter ends at zero.
"""
import pytest
import torch

from oracle import swiglu_oracle as O
from swiglu_b200 import _lib, ops

pytestmark = pytest.mark.gpu

TOL = 8e-3
DEV = "cuda"
COUNTER_WORDS = 1024  # the workspace's first 4096 bytes


@pytest.fixture(params=[2, 3], ids=["n256", "n512"])
def pair_path(request):
    _lib.set_gemm_path(request.param)
    yield
    _lib.set_gemm_path(0)
    ops.set_stream_k(True)


def _r(*shape, seed=0, scale=1.0):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(*shape, generator=g) * scale).to(torch.bfloat16)


def _workspace():
    key = (torch.cuda.current_device(), torch.cuda.current_stream().cuda_stream)
    return ops._workspaces[key]


def _run_three_ways(fn):
    """(stream-K result, second stream-K result, unsplit result); checks the
    split ran and left the counters zero."""
    fn()                                   # registers this stream's workspace
    ws = _workspace()
    ws[4096:4096 + (8 << 20)].zero_()
    a = fn()
    torch.cuda.synchronize()
    assert ws[4096:4096 + (8 << 20)].any(), "no stream-K partials were written"
    assert not ws[:4096].view(torch.int32).any(), "arrival counters not left zero"
    b = fn()
    ops.set_stream_k(False)
    try:
        c = fn()
    finally:
        ops.set_stream_k(True)
    assert ops.device_status() == 0
    return a, b, c


def _check(results, ref):
    a, b, c = [t.float().cpu() for t in results]
    assert torch.equal(a, b), "stream-K result differs between runs"
    assert O.rel_max(a, c) <= TOL
    assert O.rel_max(a, ref) <= TOL
    assert O.rel_max(c, ref) <= TOL


@pytest.mark.parametrize("a_t", [False, True])
@pytest.mark.parametrize("b_t", [False, True])
@pytest.mark.parametrize("M,N,K", [(512, 768, 2048),      # 6 (n256) or 4 (n512) tiles, all split 4 ways
                                   (2560, 4096, 512)])    # 160 / 80 tiles: full rounds + 12 / 6 split 2 ways
@pytest.mark.parametrize("out_dtype", [torch.bfloat16, torch.float32])
def test_matmul_stream_k(pair_path, a_t, b_t, M, N, K, out_dtype):
    a = _r(*((K, M) if a_t else (M, K)), seed=1)
    b = _r(*((N, K) if b_t else (K, N)), seed=2, scale=K ** -0.5)
    ref = (a.float().t() if a_t else a.float()) @ (b.float().t() if b_t else b.float())
    ad, bd = a.to(DEV), b.to(DEV)
    res = _run_three_ways(lambda: ops.matmul(ad, bd, a_t=a_t, b_t=b_t, out_dtype=out_dtype))
    _check(res, ref)


@pytest.mark.parametrize("form,layout", [(ops.W1_ROWS, O.STD), (ops.W1_T, O.PACKED)])
def test_swiglu_forward_stream_k(pair_path, form, layout):
    M, K, H = 512, 2048, 384
    x = _r(M, K, seed=5)
    w_rows_std = _r(2 * H, K, seed=6, scale=K ** -0.5)
    li, gi = O.col_index(H, layout)
    w_rows = torch.empty_like(w_rows_std)
    w_rows[li] = w_rows_std[:H]
    w_rows[gi] = w_rows_std[H:]
    w = (w_rows if form == ops.W1_ROWS else w_rows.t().contiguous()).to(DEV)
    lay = ops.LAYOUT_STD if layout == O.STD else ops.LAYOUT_PACKED128
    xd = x.to(DEV)
    res = _run_three_ways(lambda: torch.cat(ops.swiglu_fwd(xd, w, w_form=form, layout=lay,
                                                           h_from_rounded=True), dim=1))
    acc = x.float() @ w_rows.float().t()
    pre = O._round(acc, True)
    h = O.forward_logic(pre, layout, True)
    _check(res, torch.cat([pre, h], dim=1))


def test_grad_preact_stream_k(pair_path):
    M, H, Dout = 512, 768, 2048
    gy, w2 = _r(M, Dout, seed=7), _r(Dout, H, seed=8, scale=Dout ** -0.5)
    pre = _r(M, 2 * H, seed=9)
    gyd, w2d, pred = gy.to(DEV), w2.to(DEV), pre.to(DEV)
    res = _run_three_ways(lambda: ops.bwd_grad_preact_inplace(gyd, w2d, pred.clone(), layout=ops.LAYOUT_STD))
    gh = O._round(gy.float() @ w2.float(), True)
    ref = O.backward_logic(pre.float(), gh, O.STD, True)
    _check(res, ref)


def test_dw2_stream_k(pair_path):
    M, H, Dout = 4096, 512, 1024          # 4 pair tiles of 256 x 512, split 4 ways
    gy, pre = _r(M, Dout, seed=10), _r(M, 2 * H, seed=11)
    gyd, pred = gy.to(DEV), pre.to(DEV)
    res = _run_three_ways(lambda: ops.bwd_dw2(gyd, pred, layout=ops.LAYOUT_STD))
    h = O.forward_logic(pre.float(), O.STD, True)
    _check(res, gy.float().t() @ h)


def test_stale_counter_is_ignored(pair_path):
    a, b = _r(512, 2048, seed=12).to(DEV), _r(2048, 768, seed=13, scale=2048 ** -0.5).to(DEV)
    first = ops.matmul(a, b, a_t=False, b_t=False)
    ws = _workspace()
    # A launch that stopped part-way would leave counts under its own epoch.
    stale = (0x345678 << 8) | 1
    ws[:4096].view(torch.int32).fill_(stale)
    again = ops.matmul(a, b, a_t=False, b_t=False)
    torch.cuda.synchronize()
    assert torch.equal(first, again)
    counters = ws[:4096].view(torch.int32)
    # Slots this launch used are back to zero; unused ones keep the planted value.
    assert bool(((counters == 0) | (counters == stale)).all())
    assert int((counters == 0).sum()) >= 8
    ws[:4096].zero_()
    assert ops.device_status() == 0
