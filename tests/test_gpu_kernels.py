"""Each native entry point against the CPU oracle on the same seeded inputs.

GPU only. bf16 results are compared with a CPU fp32 computation from the same
bf16 values, rounded to bf16 at the points the reference rounds; the bound is
rel_max <= 8e-3 (one bf16 ulp is 2^-8 = 3.9e-3 of the element; rel_max is
relative to the largest element). f32 results: rel_max <= 1e-5.
"""
import pytest
import torch

from oracle import swiglu_oracle as O
from swiglu_b200 import _lib, ops

pytestmark = pytest.mark.gpu

BF16_TOL = 8e-3
F32_TOL = 1e-5
DEV = "cuda"


@pytest.fixture(params=[1, 2, 3], ids=["1sm", "2sm", "2sm_n512"])
def gemm_path(request):
    """Run the bf16 GEMMs on the single-SM kernel and on the 2-SM (CTA pair) kernel."""
    _lib.set_gemm_path(request.param)
    yield request.param
    _lib.set_gemm_path(0)


def _r(*shape, seed=0, scale=1.0, dtype=torch.bfloat16):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(*shape, generator=g) * scale).to(dtype)


def _tol(dtype):
    return BF16_TOL if dtype == torch.bfloat16 else F32_TOL


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("a_t", [False, True])
@pytest.mark.parametrize("b_t", [False, True])
@pytest.mark.parametrize("M,N,K", [(256, 512, 256), (200, 264, 136), (128, 256, 64), (384, 768, 1024),
                                   (1000, 520, 328)])
def test_matmul_layouts(gemm_path, dtype, a_t, b_t, M, N, K):
    if a_t and M % 8:
        pytest.skip("MN-major A needs M % 8 == 0")
    a = _r(*((K, M) if a_t else (M, K)), seed=1, dtype=dtype)
    b = _r(*((N, K) if b_t else (K, N)), seed=2, scale=K ** -0.5, dtype=dtype)
    ref = (a.float().t() if a_t else a.float()) @ (b.float().t() if b_t else b.float())
    out = ops.matmul(a.to(DEV), b.to(DEV), a_t=a_t, b_t=b_t)
    assert out.dtype == dtype
    assert O.rel_max(out.cpu(), ref) <= _tol(dtype)


def test_matmul_f32_output_of_bf16_gemm(gemm_path):
    a, b = _r(256, 512, seed=3), _r(512, 256, seed=4, scale=512 ** -0.5)
    ref = a.float() @ b.float()
    out = ops.matmul(a.to(DEV), b.to(DEV), a_t=False, b_t=False, out_dtype=torch.float32)
    assert out.dtype == torch.float32
    assert O.rel_max(out.cpu(), ref) <= 1e-5


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("form,layout", [(ops.W1_ROWS, O.STD), (ops.W1_T, O.STD), (ops.W1_T, O.PACKED)])
@pytest.mark.parametrize("rounded", [False, True])
@pytest.mark.parametrize("M,K,H", [(256, 256, 256), (200, 136, 384), (128, 64, 128), (640, 192, 512)])
def test_swiglu_forward_epilogue(gemm_path, dtype, form, layout, rounded, M, K, H):
    if layout == O.PACKED and H % 128:
        pytest.skip("packed layout needs H % 128 == 0")
    x = _r(M, K, seed=5, dtype=dtype)
    w_rows_std = _r(2 * H, K, seed=6, scale=K ** -0.5, dtype=dtype)          # [left; gate] rows
    li, gi = O.col_index(H, layout)
    w_rows = torch.empty_like(w_rows_std)
    w_rows[li] = w_rows_std[:H]
    w_rows[gi] = w_rows_std[H:]
    w = w_rows if form == ops.W1_ROWS else w_rows.t().contiguous()
    lay = ops.LAYOUT_STD if layout == O.STD else ops.LAYOUT_PACKED128
    preact, h = ops.swiglu_fwd(x.to(DEV), w.to(DEV), w_form=form, layout=lay, h_from_rounded=rounded)
    bf = dtype == torch.bfloat16
    acc = x.float() @ w_rows.float().t()
    ref_pre = O._round(acc, bf)
    ref_h = O.forward_logic(ref_pre if (rounded and bf) else acc, layout, bf)
    assert O.rel_max(preact.cpu(), ref_pre) <= _tol(dtype)
    assert O.rel_max(h.cpu(), ref_h) <= _tol(dtype)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("layout", [O.STD, O.PACKED])
@pytest.mark.parametrize("M,H,Dout", [(256, 256, 128), (200, 384, 136), (1000, 128, 256), (333, 640, 600)])
def test_dw2_with_recomputed_h(gemm_path, dtype, layout, M, H, Dout):
    lay = ops.LAYOUT_STD if layout == O.STD else ops.LAYOUT_PACKED128
    gy = _r(M, Dout, seed=7, dtype=dtype)
    preact = _r(M, 2 * H, seed=8, dtype=dtype)
    bf = dtype == torch.bfloat16
    h = O.forward_logic(preact.float(), layout, bf)
    ref = gy.float().t() @ h
    out = ops.bwd_dw2(gy.to(DEV), preact.to(DEV), layout=lay)
    assert O.rel_max(out.cpu(), ref) <= _tol(dtype)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("layout", [O.STD, O.PACKED])
@pytest.mark.parametrize("M,H,Dout", [(256, 256, 128), (200, 384, 136), (128, 640, 64), (700, 512, 200)])
def test_grad_preact_inplace(gemm_path, dtype, layout, M, H, Dout):
    lay = ops.LAYOUT_STD if layout == O.STD else ops.LAYOUT_PACKED128
    gy = _r(M, Dout, seed=9, dtype=dtype)
    w2 = _r(Dout, H, seed=10, scale=H ** -0.5, dtype=dtype)
    preact = _r(M, 2 * H, seed=11, dtype=dtype)
    bf = dtype == torch.bfloat16
    grad_h = O._round(gy.float() @ w2.float(), bf)
    ref = O.backward_logic(preact.float(), grad_h, layout, bf)
    p_dev = preact.to(DEV)
    ptr = p_dev.data_ptr()
    out = ops.bwd_grad_preact_inplace(gy.to(DEV), w2.to(DEV), p_dev, layout=lay)
    assert out.data_ptr() == ptr
    assert O.rel_max(p_dev.cpu(), ref) <= _tol(dtype)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("layout", [O.STD, O.PACKED])
@pytest.mark.parametrize("M,H,Dout", [(256, 256, 128), (200, 384, 136), (700, 512, 200), (1024, 768, 640)])
def test_grad_preact_inplace_emit_h(gemm_path, dtype, layout, M, H, Dout):
    """The emit-h form writes the same grad_preact as the plain call, h of the
    replaced preact within the bound, and dW2 = grad_y^T h from it matches the
    prologue dW2 kernel and the oracle."""
    lay = ops.LAYOUT_STD if layout == O.STD else ops.LAYOUT_PACKED128
    gy = _r(M, Dout, seed=12, dtype=dtype).to(DEV)
    w2 = _r(Dout, H, seed=13, scale=Dout ** -0.5, dtype=dtype).to(DEV)
    preact = _r(M, 2 * H, seed=14, dtype=dtype)
    bf = dtype == torch.bfloat16
    ref_h = O.forward_logic(preact.float(), layout, bf)
    dw2_prologue = ops.bwd_dw2(gy, preact.to(DEV), layout=lay)
    plain = ops.bwd_grad_preact_inplace(gy, w2, preact.to(DEV), layout=lay)
    h = torch.empty((M, H), dtype=dtype, device=DEV)
    gp = ops.bwd_grad_preact_inplace(gy, w2, preact.to(DEV), layout=lay, h_out=h)
    assert torch.equal(gp, plain)
    assert O.rel_max(h.cpu(), ref_h) <= _tol(dtype)
    if bf:
        assert O.bf16_ulps(h.cpu(), ref_h).max().item() <= 1
    dw2 = ops.matmul(gy, h, a_t=True, b_t=False)
    ref_dw2 = gy.cpu().float().t() @ ref_h
    assert O.rel_max(dw2.cpu(), ref_dw2) <= _tol(dtype)
    assert O.rel_max(dw2.cpu(), dw2_prologue.cpu().float()) <= _tol(dtype)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("layout", [O.STD, O.PACKED])
def test_pointwise_kernels(dtype, layout):
    lay = ops.LAYOUT_STD if layout == O.STD else ops.LAYOUT_PACKED128
    M, H = 300, 512
    preact = _r(M, 2 * H, seed=12, dtype=dtype)
    gh = _r(M, H, seed=13, dtype=dtype)
    bf = dtype == torch.bfloat16
    h = ops.forward_logic(preact.to(DEV), layout=lay)
    ref_h = O.forward_logic(preact, layout, bf)
    assert O.rel_max(h.cpu(), ref_h) <= _tol(dtype)
    gp = ops.backward_logic(preact.to(DEV), gh.to(DEV), layout=lay)
    ref_gp = O.backward_logic(preact, gh, layout, bf)
    assert O.rel_max(gp.cpu(), ref_gp) <= _tol(dtype)
    if bf:
        # Each bf16 element is one f32 chain rounded once, as Inductor's fused
        # pointwise kernel does: it may differ from the oracle's only where the
        # f32 values (fast exp/reciprocal vs torch.sigmoid) straddle a rounding
        # boundary, i.e. by at most one bf16 ulp, element by element.
        assert O.bf16_ulps(h.cpu(), ref_h).max().item() <= 1
        assert O.bf16_ulps(gp.cpu(), ref_gp).max().item() <= 1


@pytest.mark.parametrize("layout", [O.STD, O.PACKED])
def test_pointwise_kernels_wide_range_ulps(layout):
    """Every bf16 value class the gate can take (large negative, tiny,
    subnormal, large positive) through the pointwise kernels: at most one bf16
    ulp from the oracle per element."""
    lay = ops.LAYOUT_STD if layout == O.STD else ops.LAYOUT_PACKED128
    M, H = 512, 256
    g = torch.Generator().manual_seed(31)
    mag = torch.exp2(torch.empty(M, 2 * H).uniform_(-20, 6, generator=g))
    sign = torch.where(torch.rand(M, 2 * H, generator=g) < 0.5, -1.0, 1.0)
    preact = (mag * sign).to(torch.bfloat16)
    gh = torch.randn(M, H, generator=g).to(torch.bfloat16)
    h = ops.forward_logic(preact.to(DEV), layout=lay)
    gp = ops.backward_logic(preact.to(DEV), gh.to(DEV), layout=lay)
    assert O.bf16_ulps(h.cpu(), O.forward_logic(preact, layout, True)).max().item() <= 1
    assert O.bf16_ulps(gp.cpu(), O.backward_logic(preact, gh, layout, True)).max().item() <= 1


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("block", [128, 64, 32])
def test_pack_unpack_exact(dtype, block):
    w = _r(48, 2 * 256, seed=14, dtype=dtype)
    pk = ops.pack_chunked(w.to(DEV), block, unpack=False)
    assert torch.equal(pk.cpu(), O.pack_weight_chunked(w, block))
    assert torch.equal(ops.pack_chunked(pk, block, unpack=True).cpu(), w)


def test_empty_batch_is_a_no_op_with_zero_weight_grads():
    H, D, Dout = 128, 64, 64
    x = torch.empty(0, D, dtype=torch.bfloat16, device=DEV)
    w1 = _r(2 * H, D, seed=15).to(DEV)
    preact, h = ops.swiglu_fwd(x, w1, w_form=ops.W1_ROWS, layout=ops.LAYOUT_STD, h_from_rounded=True)
    assert preact.shape == (0, 2 * H) and h.shape == (0, H)
    gy = torch.empty(0, Dout, dtype=torch.bfloat16, device=DEV)
    dw2 = ops.bwd_dw2(gy, preact, layout=ops.LAYOUT_STD)
    assert dw2.shape == (Dout, H) and dw2.abs().max().item() == 0.0


def test_device_status_healthy_after_all_kernels():
    assert ops.device_status(0) == 0


@pytest.mark.parametrize("a_t,b_t", [(True, False), (False, False), (False, True)])
def test_matmul_tile_width_hint(a_t, b_t):
    """tile_n=512 under the default path selection: a shape with more than a
    wave of CTA pairs takes the 256 x 512 kernel; the result matches the
    default tiles within the bf16 bound, and invalid widths are rejected."""
    M, N, K = 2048, 3584, 1536
    a = _r(*((K, M) if a_t else (M, K)), seed=21)
    b = _r(*((N, K) if b_t else (K, N)), seed=22, scale=K ** -0.5)
    ref = (a.float().t() if a_t else a.float()) @ (b.float().t() if b_t else b.float())
    ad, bd = a.to(DEV), b.to(DEV)
    wide = ops.matmul(ad, bd, a_t=a_t, b_t=b_t, tile_n=512)
    narrow = ops.matmul(ad, bd, a_t=a_t, b_t=b_t)
    assert O.rel_max(wide.cpu(), ref) <= BF16_TOL
    assert O.rel_max(wide.cpu(), narrow.cpu().float()) <= BF16_TOL
    with pytest.raises(_lib.SwigluError):
        ops.matmul(ad, bd, a_t=a_t, b_t=b_t, tile_n=384)


@pytest.mark.parametrize("path", [2, 3], ids=["n256", "n512"])
@pytest.mark.parametrize("form,layout", [(ops.W1_ROWS, O.STD), (ops.W1_T, O.PACKED)])
@pytest.mark.parametrize("want_preact", [True, False])
def test_swiglu_forward_tma_epilogue(path, form, layout, want_preact):
    """M >= 4096 with H % 32 == 0 takes the 2-SM kernel's TMA-store SwiGLU
    epilogue (preact and h staged in shared memory); checked against the
    oracle, and the h-only form against the full one bit for bit."""
    M, K, H = 4096, 256, 640
    x = _r(M, K, seed=31)
    w_rows_std = _r(2 * H, K, seed=32, scale=K ** -0.5)
    li, gi = O.col_index(H, layout)
    w_rows = torch.empty_like(w_rows_std)
    w_rows[li] = w_rows_std[:H]
    w_rows[gi] = w_rows_std[H:]
    w = (w_rows if form == ops.W1_ROWS else w_rows.t().contiguous()).to(DEV)
    lay = ops.LAYOUT_STD if layout == O.STD else ops.LAYOUT_PACKED128
    _lib.set_gemm_path(path)
    try:
        full_pre, full_h = ops.swiglu_fwd(x.to(DEV), w, w_form=form, layout=lay, h_from_rounded=True)
        pre, h = ops.swiglu_fwd(x.to(DEV), w, w_form=form, layout=lay, h_from_rounded=True,
                                want_preact=want_preact)
    finally:
        _lib.set_gemm_path(0)
    acc = x.float() @ w_rows.float().t()
    ref_pre = O._round(acc, True)
    ref_h = O.forward_logic(ref_pre, layout, True)
    assert O.rel_max(full_pre.cpu(), ref_pre) <= BF16_TOL
    assert O.rel_max(full_h.cpu(), ref_h) <= BF16_TOL
    assert torch.equal(h, full_h)
    assert (pre is None) == (not want_preact)


def test_swiglu_forward_wide_tiles_by_size():
    """At K >= 8192 (and 8 waves of tiles) the size rule runs GEMM1 + SwiGLU on
    256 x 512 pair tiles. Each output still sums its k-blocks in the same
    order as on 256 x 256 tiles (neither launch splits a tail here), so the
    bits agree; sampled rows against the f64 product."""
    M = K = H = 8192
    assert _lib.swiglu_fwd_plan(M, K, H, torch.cuda.get_device_properties(0).multi_processor_count) == 3
    x = _r(M, K, seed=11)
    w = _r(2 * H, K, seed=12, scale=K ** -0.5)
    xd, wd = x.to(DEV), w.to(DEV)
    pre_w, h_w = ops.swiglu_fwd(xd, wd, w_form=ops.W1_ROWS, layout=ops.LAYOUT_STD, h_from_rounded=True)
    _lib.set_gemm_path(2)
    try:
        pre_n, h_n = ops.swiglu_fwd(xd, wd, w_form=ops.W1_ROWS, layout=ops.LAYOUT_STD, h_from_rounded=True)
    finally:
        _lib.set_gemm_path(0)
    assert torch.equal(pre_w, pre_n) and torch.equal(h_w, h_n)
    rows = torch.tensor([0, 1, 255, 256, 511, 4095, 4096, 8191])
    ref_pre = O._round(x[rows].double() @ w.double().t(), True)
    ref_h = O.forward_logic(ref_pre, O.STD, True)
    assert O.rel_max(pre_w[rows.to(DEV)].cpu().double(), ref_pre) <= BF16_TOL
    assert O.rel_max(h_w[rows.to(DEV)].cpu().double(), ref_h) <= BF16_TOL
    assert ops.device_status(0) == 0


def test_grad_preact_wide_tiles_by_size():
    """grad_h + dSwiGLU with K = Dout >= 8192 (and 8 waves of tiles) runs on
    256 x 512 pair tiles by size. That launch splits its last round of tiles
    along K (stream-K: 768 tiles on 74 pairs) where the 256 x 256 launch
    does not, so the two agree to the bf16 rounding of the f32 sums, not bit
    for bit; both against the oracle's f64 chain on sampled rows."""
    M, H, Dout = 8192, 12288, 8192
    gy = _r(M, Dout, seed=21)
    w2 = _r(Dout, H, seed=22, scale=Dout ** -0.5)
    preact = _r(M, 2 * H, seed=23)
    gyd, w2d = gy.to(DEV), w2.to(DEV)
    outs = {}
    for path in (0, 2):
        _lib.set_gemm_path(path)
        try:
            p_dev = preact.to(DEV)
            h = torch.empty((M, H), dtype=torch.bfloat16, device=DEV)
            ops.bwd_grad_preact_inplace(gyd, w2d, p_dev, layout=ops.LAYOUT_STD, h_out=h)
            outs[path] = (p_dev, h)
        finally:
            _lib.set_gemm_path(0)
    for a, b in zip(outs[0], outs[2]):
        assert ((a.float() - b.float()).abs().max() / b.float().abs().max()).item() <= BF16_TOL
    rows = torch.tensor([0, 1, 255, 256, 4095, 8191, *range(7936, 8192, 37)])
    grad_h = O._round(gy[rows].double() @ w2.double(), True)
    ref = O.backward_logic(preact[rows].double(), grad_h, O.STD, True)
    ref_h = O.forward_logic(preact[rows].double(), O.STD, True)
    for gp, h in outs.values():
        assert O.rel_max(gp[rows.to(DEV)].cpu().double(), ref) <= BF16_TOL
        assert O.bf16_ulps(h[rows.to(DEV)].cpu(), ref_h).max().item() <= 1
    assert ops.device_status(0) == 0
