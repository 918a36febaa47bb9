"""torch.library registration of the native entry points, so the recompute
Functions compose under torch.compile.

Each op is opaque to the compiler: a fake (shape-only) implementation
describes its outputs, and the real one calls libswiglu_b200.so through
`swiglu_b200.ops`. The in-place grad_h op declares what it writes (preact,
and h when given), so functionalization and Inductor's re-inplacing see the
mutation. The recompute Functions call `kernels()`: these ops while Dynamo
traces, the plain `ops` functions in eager mode (no dispatcher overhead).

This is the composability item of the reference's fair-compile comparison
(bench_fair_compile.py:45, torch.compile of the standard MLP as the
baseline): with these ops a compiled stack of SwiGLUMLPCustom blocks traces
without graph breaks and runs the same kernels as eager.
"""
from __future__ import annotations

from typing import Optional

import torch

from . import ops
from .ops import W1_ROWS

_NS = "swiglu_b200"


def _n2(w: torch.Tensor, w_form: int) -> int:
    return w.shape[0] if w_form == W1_ROWS else w.shape[1]


@torch.library.custom_op(f"{_NS}::swiglu_fwd", mutates_args=(), device_types="cuda")
def swiglu_fwd(x: torch.Tensor, w: torch.Tensor, w_form: int, layout: int, h_from_rounded: bool,
               group_size_m: int) -> tuple[torch.Tensor, torch.Tensor]:
    """(preact [M, 2H], h [M, H]) in one launch."""
    return ops.swiglu_fwd(x, w, w_form=w_form, layout=layout, h_from_rounded=h_from_rounded,
                          group_size_m=group_size_m)


@swiglu_fwd.register_fake
def _(x, w, w_form, layout, h_from_rounded, group_size_m):
    n2 = _n2(w, w_form)
    return x.new_empty((x.shape[0], n2)), x.new_empty((x.shape[0], n2 // 2))


@torch.library.custom_op(f"{_NS}::swiglu_fwd_h", mutates_args=(), device_types="cuda")
def swiglu_fwd_h(x: torch.Tensor, w: torch.Tensor, w_form: int, layout: int, h_from_rounded: bool,
                 group_size_m: int) -> torch.Tensor:
    """h [M, H] only (the no-save forward)."""
    return ops.swiglu_fwd(x, w, w_form=w_form, layout=layout, h_from_rounded=h_from_rounded,
                          want_preact=False, group_size_m=group_size_m)[1]


@swiglu_fwd_h.register_fake
def _(x, w, w_form, layout, h_from_rounded, group_size_m):
    return x.new_empty((x.shape[0], _n2(w, w_form) // 2))


@torch.library.custom_op(f"{_NS}::swiglu_fwd_preact", mutates_args=(), device_types="cuda")
def swiglu_fwd_preact(x: torch.Tensor, w: torch.Tensor, w_form: int, layout: int,
                      group_size_m: int) -> torch.Tensor:
    """preact [M, 2H] only (the full-checkpoint backward's recompute)."""
    return ops.swiglu_fwd(x, w, w_form=w_form, layout=layout, h_from_rounded=True, want_h=False,
                          group_size_m=group_size_m)[0]


@swiglu_fwd_preact.register_fake
def _(x, w, w_form, layout, group_size_m):
    return x.new_empty((x.shape[0], _n2(w, w_form)))


@torch.library.custom_op(f"{_NS}::matmul", mutates_args=(), device_types="cuda")
def matmul(a: torch.Tensor, b: torch.Tensor, a_t: bool, b_t: bool, tile_n: int) -> torch.Tensor:
    """op(a) . op(b) in a's dtype (tile_n: preferred 2-SM tile width, 0 = default)."""
    return ops.matmul(a, b, a_t=a_t, b_t=b_t, tile_n=tile_n)


@matmul.register_fake
def _(a, b, a_t, b_t, tile_n):
    m = a.shape[1] if a_t else a.shape[0]
    n = b.shape[0] if b_t else b.shape[1]
    return a.new_empty((m, n))


@torch.library.custom_op(f"{_NS}::bwd_dw2", mutates_args=(), device_types="cuda")
def bwd_dw2(grad_y: torch.Tensor, preact: torch.Tensor, layout: int) -> torch.Tensor:
    """dW2 [Dout, H] with h recomputed in the operand prologue."""
    return ops.bwd_dw2(grad_y, preact, layout=layout)


@bwd_dw2.register_fake
def _(grad_y, preact, layout):
    return grad_y.new_empty((grad_y.shape[1], preact.shape[1] // 2))


@torch.library.custom_op(f"{_NS}::bwd_grad_preact_", mutates_args=("preact", "h_out"), device_types="cuda")
def bwd_grad_preact_(grad_y: torch.Tensor, w2: torch.Tensor, preact: torch.Tensor, layout: int,
                     h_out: Optional[torch.Tensor]) -> None:
    """preact <- grad_preact in place (and h_out <- h of the replaced preact)."""
    ops.bwd_grad_preact_inplace(grad_y, w2, preact, layout=layout, h_out=h_out)


@bwd_grad_preact_.register_fake
def _(grad_y, w2, preact, layout, h_out):
    return None


@torch.library.custom_op(f"{_NS}::quantize_e4m3", mutates_args=(), device_types="cuda")
def quantize_e4m3(t: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """(q e4m3 [R, C], row scales [R]) of a bf16 [R, C] matrix."""
    return ops.quantize_rows_e4m3(t)


@quantize_e4m3.register_fake
def _(t):
    return t.new_empty(t.shape, dtype=torch.float8_e4m3fn), t.new_empty((t.shape[0],), dtype=torch.float32)


@torch.library.custom_op(f"{_NS}::swiglu_fwd_e4m3", mutates_args=(), device_types="cuda")
def swiglu_fwd_e4m3(xq: torch.Tensor, xs: torch.Tensor, wq: torch.Tensor, ws: torch.Tensor,
                    layout: int) -> tuple[torch.Tensor, torch.Tensor]:
    """(preact [M, 2H], h [M, H]) in bf16 from e4m3 x and W1 rows."""
    return ops.swiglu_fwd_e4m3(xq, xs, wq, ws, layout=layout, h_from_rounded=True)


@swiglu_fwd_e4m3.register_fake
def _(xq, xs, wq, ws, layout):
    m, n2 = xq.shape[0], wq.shape[0]
    return (xq.new_empty((m, n2), dtype=torch.bfloat16), xq.new_empty((m, n2 // 2), dtype=torch.bfloat16))


@torch.library.custom_op(f"{_NS}::swiglu_fwd_e4m3_h", mutates_args=(), device_types="cuda")
def swiglu_fwd_e4m3_h(xq: torch.Tensor, xs: torch.Tensor, wq: torch.Tensor, ws: torch.Tensor,
                      layout: int) -> torch.Tensor:
    """h [M, H] only (the no-save e4m3 forward)."""
    return ops.swiglu_fwd_e4m3(xq, xs, wq, ws, layout=layout, h_from_rounded=True, want_preact=False)[1]


@swiglu_fwd_e4m3_h.register_fake
def _(xq, xs, wq, ws, layout):
    return xq.new_empty((xq.shape[0], wq.shape[0] // 2), dtype=torch.bfloat16)


@torch.library.custom_op(f"{_NS}::matmul_e4m3", mutates_args=(), device_types="cuda")
def matmul_e4m3(aq: torch.Tensor, a_scale: torch.Tensor, bq: torch.Tensor, b_scale: torch.Tensor) -> torch.Tensor:
    """A . B^T in bf16 for e4m3 A [M, K], B [N, K] with their row scales."""
    return ops.matmul_e4m3(aq, a_scale, bq, b_scale)


@matmul_e4m3.register_fake
def _(aq, a_scale, bq, b_scale):
    return aq.new_empty((aq.shape[0], bq.shape[0]), dtype=torch.bfloat16)


class _Eager:
    """The calls the Functions make, on the plain ops functions."""

    @staticmethod
    def swiglu_fwd(x, w, w_form, layout, h_from_rounded, group_size_m=ops.DEFAULT_GROUP_M):
        return ops.swiglu_fwd(x, w, w_form=w_form, layout=layout, h_from_rounded=h_from_rounded,
                              group_size_m=group_size_m)

    @staticmethod
    def swiglu_fwd_h(x, w, w_form, layout, h_from_rounded, group_size_m=ops.DEFAULT_GROUP_M):
        return ops.swiglu_fwd(x, w, w_form=w_form, layout=layout, h_from_rounded=h_from_rounded,
                              want_preact=False, group_size_m=group_size_m)[1]

    @staticmethod
    def swiglu_fwd_preact(x, w, w_form, layout, group_size_m=ops.DEFAULT_GROUP_M):
        return ops.swiglu_fwd(x, w, w_form=w_form, layout=layout, h_from_rounded=True, want_h=False,
                              group_size_m=group_size_m)[0]

    @staticmethod
    def matmul(a, b, a_t, b_t, tile_n=0):
        return ops.matmul(a, b, a_t=a_t, b_t=b_t, tile_n=tile_n)

    @staticmethod
    def bwd_dw2(grad_y, preact, layout):
        return ops.bwd_dw2(grad_y, preact, layout=layout)

    @staticmethod
    def bwd_grad_preact_(grad_y, w2, preact, layout, h_out=None):
        ops.bwd_grad_preact_inplace(grad_y, w2, preact, layout=layout, h_out=h_out)

    @staticmethod
    def quantize_e4m3(t):
        return ops.quantize_rows_e4m3(t)

    @staticmethod
    def swiglu_fwd_e4m3(xq, xs, wq, ws, layout):
        return ops.swiglu_fwd_e4m3(xq, xs, wq, ws, layout=layout, h_from_rounded=True)

    @staticmethod
    def swiglu_fwd_e4m3_h(xq, xs, wq, ws, layout):
        return ops.swiglu_fwd_e4m3(xq, xs, wq, ws, layout=layout, h_from_rounded=True, want_preact=False)[1]

    @staticmethod
    def matmul_e4m3(aq, a_scale, bq, b_scale):
        return ops.matmul_e4m3(aq, a_scale, bq, b_scale)


class _Traced:
    """The same calls as registered ops (what Dynamo records)."""

    @staticmethod
    def swiglu_fwd(x, w, w_form, layout, h_from_rounded, group_size_m=ops.DEFAULT_GROUP_M):
        return torch.ops.swiglu_b200.swiglu_fwd(x, w, w_form, layout, h_from_rounded, group_size_m)

    @staticmethod
    def swiglu_fwd_h(x, w, w_form, layout, h_from_rounded, group_size_m=ops.DEFAULT_GROUP_M):
        return torch.ops.swiglu_b200.swiglu_fwd_h(x, w, w_form, layout, h_from_rounded, group_size_m)

    @staticmethod
    def swiglu_fwd_preact(x, w, w_form, layout, group_size_m=ops.DEFAULT_GROUP_M):
        return torch.ops.swiglu_b200.swiglu_fwd_preact(x, w, w_form, layout, group_size_m)

    @staticmethod
    def matmul(a, b, a_t, b_t, tile_n=0):
        return torch.ops.swiglu_b200.matmul(a, b, a_t, b_t, tile_n)

    @staticmethod
    def bwd_dw2(grad_y, preact, layout):
        return torch.ops.swiglu_b200.bwd_dw2(grad_y, preact, layout)

    @staticmethod
    def bwd_grad_preact_(grad_y, w2, preact, layout, h_out=None):
        torch.ops.swiglu_b200.bwd_grad_preact_(grad_y, w2, preact, layout, h_out)

    @staticmethod
    def quantize_e4m3(t):
        return torch.ops.swiglu_b200.quantize_e4m3(t)

    @staticmethod
    def swiglu_fwd_e4m3(xq, xs, wq, ws, layout):
        return torch.ops.swiglu_b200.swiglu_fwd_e4m3(xq, xs, wq, ws, layout)

    @staticmethod
    def swiglu_fwd_e4m3_h(xq, xs, wq, ws, layout):
        return torch.ops.swiglu_b200.swiglu_fwd_e4m3_h(xq, xs, wq, ws, layout)

    @staticmethod
    def matmul_e4m3(aq, a_scale, bq, b_scale):
        return torch.ops.swiglu_b200.matmul_e4m3(aq, a_scale, bq, b_scale)


def kernels():
    """The registered ops while torch.compile traces, else the eager calls."""
    return _Traced if torch.compiler.is_compiling() else _Eager
