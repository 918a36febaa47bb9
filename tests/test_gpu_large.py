"""64-bit addressing: one block whose preact holds more than 2^31 elements.

The tensor-parallel configuration (M=65536, D=8192, H=28672) gives every
rank at t=1 a preact of 65536 x 57344 = 3.76e9 elements, beyond any 32-bit
element or byte offset. Here K and Dout are small so the GEMMs are cheap, but
M x 2H = 65536 x 34816 = 2.28e9 elements (4.56 GB) crosses both the 2^31-byte
(row 30840) and the 2^31-element (row 61680) boundaries. Rows and columns on
both sides of them are checked against the CPU oracle for every stage:
GEMM1 + SwiGLU epilogue (preact, h), dW2 with h recomputed from preact,
grad_preact in place with h emitted, dx, dW1 and dW2 from the emitted h.
Bound as in the other bf16 kernel tests: rel_max <= 8e-3.
"""
import pytest
import torch

from oracle import swiglu_oracle as O
from swiglu_b200 import _lib, ops

pytestmark = pytest.mark.gpu

BF16_TOL = 8e-3
DEV = "cuda"
M, D, H, DOUT = 65536, 64, 17408, 128


def _r(*shape, seed, scale=1.0):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(*shape, generator=g) * scale).to(torch.bfloat16)


def _rows():
    n2 = 2 * H
    byte_edge = (1 << 31) // (2 * n2)   # first row past 2^31 bytes of preact
    elem_edge = (1 << 31) // n2         # first row past 2^31 elements
    assert M * n2 > (1 << 31) and 0 < byte_edge < elem_edge < M - 64
    spans = [(0, 32), (byte_edge - 16, byte_edge + 16), (elem_edge - 32, elem_edge + 32), (M - 32, M)]
    return torch.cat([torch.arange(a, b) for a, b in spans])


@pytest.mark.parametrize("path", [1, 2, 3], ids=["1sm", "2sm", "2sm_n512"])
def test_block_with_preact_beyond_2g_elements(path):
    _lib.set_gemm_path(path)
    try:
        x, w1 = _r(M, D, seed=40), _r(2 * H, D, seed=41, scale=D ** -0.5)
        w2, gy = _r(DOUT, H, seed=42, scale=H ** -0.5), _r(M, DOUT, seed=43)
        xd, w1d, w2d, gyd = (t.to(DEV) for t in (x, w1, w2, gy))
        rows = _rows()
        rows_d = rows.to(DEV)
        cols = torch.cat([torch.arange(0, 32), torch.arange(H // 2 - 16, H // 2 + 16), torch.arange(H - 32, H)])
        cols_d = cols.to(DEV)

        # forward: preact and h on the sampled rows
        preact, h = ops.swiglu_fwd(xd, w1d, w_form=ops.W1_ROWS, layout=ops.LAYOUT_STD, h_from_rounded=True)
        pre_rows = preact.index_select(0, rows_d).cpu()
        ref_pre = O._round(x[rows].float() @ w1.float().t(), True)
        assert O.rel_max(pre_rows, ref_pre) <= BF16_TOL
        assert O.rel_max(h.index_select(0, rows_d).cpu(), O.forward_logic(ref_pre, O.STD, True)) <= BF16_TOL

        # dW2 with h recomputed from preact, on the sampled hidden units
        pre_cols = torch.cat([preact.index_select(1, cols_d), preact.index_select(1, cols_d + H)], dim=1).cpu()
        h_cols = O.forward_logic(pre_cols.float(), O.STD, True)
        dw2_pro = ops.bwd_dw2(gyd, preact, layout=ops.LAYOUT_STD)
        ref_dw2 = gy.float().t() @ h_cols
        assert O.rel_max(dw2_pro.index_select(1, cols_d).cpu(), ref_dw2) <= BF16_TOL

        # grad_preact in place, h emitted into the forward's h buffer
        gp = ops.bwd_grad_preact_inplace(gyd, w2d, preact, layout=ops.LAYOUT_STD, h_out=h)
        assert gp.data_ptr() == preact.data_ptr()
        grad_h = O._round(gy[rows].float() @ w2.float(), True)
        ref_gp = O.backward_logic(pre_rows.float(), grad_h, O.STD, True)
        assert O.rel_max(gp.index_select(0, rows_d).cpu(), ref_gp) <= BF16_TOL
        assert O.rel_max(h.index_select(0, rows_d).cpu(), O.forward_logic(pre_rows.float(), O.STD, True)) \
            <= BF16_TOL

        # dx = grad_preact . W1 on the sampled rows (K = 2H)
        dx = ops.matmul(gp, w1d, a_t=False, b_t=False)
        ref_dx = gp.index_select(0, rows_d).cpu().float() @ w1.float()
        assert O.rel_max(dx.index_select(0, rows_d).cpu(), ref_dx) <= BF16_TOL

        # dW1 = grad_preact^T . x on sampled left and gate rows (K = M)
        gcols_d = torch.cat([cols_d, cols_d + H])
        dw1 = ops.matmul(gp, xd, a_t=True, b_t=False, tile_n=512)
        ref_dw1 = gp.index_select(1, gcols_d).cpu().float().t() @ x.float()
        assert O.rel_max(dw1.index_select(0, gcols_d).cpu(), ref_dw1) <= BF16_TOL

        # dW2 = grad_y^T . h from the emitted h (K = M)
        dw2 = ops.matmul(gyd, h, a_t=True, b_t=False)
        ref_dw2e = gy.float().t() @ h.index_select(1, cols_d).cpu().float()
        assert O.rel_max(dw2.index_select(1, cols_d).cpu(), ref_dw2e) <= BF16_TOL
        assert ops.device_status(0) == 0
    finally:
        _lib.set_gemm_path(0)


@pytest.mark.parametrize("M,N,K,a_t,b_t", [(65536, 2048, 64, False, True), (4096, 20480, 64, True, False)],
                         ids=["y_form", "dw2_form"])
def test_matmul_size_rule_takes_wide_tiles(M, N, K, a_t, b_t):
    """Plain GEMMs with no width preference whose 256 x 512 tiles make at
    least 8 waves of CTA pairs (1024 and 640 tiles here) run on those tiles;
    the result matches the CPU product and the 256-column tiles within the bound."""
    a = _r(*((K, M) if a_t else (M, K)), seed=44)
    b = _r(*((N, K) if b_t else (K, N)), seed=45, scale=K ** -0.5)
    ad, bd = a.to(DEV), b.to(DEV)
    rows = torch.cat([torch.arange(0, 64), torch.arange(M // 2, M // 2 + 64), torch.arange(M - 64, M)])
    op_a = (a.t() if a_t else a)[rows].float()
    ref = op_a @ (b.t() if b_t else b).float()
    auto = ops.matmul(ad, bd, a_t=a_t, b_t=b_t)
    narrow = ops.matmul(ad, bd, a_t=a_t, b_t=b_t, tile_n=256)
    rows_d = rows.to(DEV)
    assert O.rel_max(auto.index_select(0, rows_d).cpu(), ref) <= BF16_TOL
    assert O.rel_max(auto.cpu(), narrow.cpu().float()) <= BF16_TOL
    assert ops.device_status(0) == 0
