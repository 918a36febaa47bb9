"""torch.library registration of the native ops (no GPU needed).

The recompute Functions are traced with fake tensors through the registered
ops (the path torch.compile takes): the forward+backward graph must hold only
this library's ops plus views and the h buffer, with the in-place grad_h op
recorded as a mutation of preact; output shapes come from the fake
implementations. A registered op called on real CPU tensors must fail (there
is no CPU kernel behind the product path).
"""
import pytest
import torch
from torch.fx.experimental.proxy_tensor import make_fx

import fused_forward as FF
import fused_forward_packed as FP
import swiglu_recompute as SR
from swiglu_b200 import library, ops

M, D, H, Dout = 256, 128, 256, 64


@pytest.fixture
def traced(monkeypatch):
    """Route the Functions through the registered ops, as under Dynamo."""
    monkeypatch.setattr(library, "kernels", lambda: library._Traced)
    for mod in (SR, FF, FP):
        monkeypatch.setattr(mod, "kernels", lambda: library._Traced)
    default = ops.dw2_mode()
    yield
    ops.set_dw2_mode(default)


def _trace(fn, w1_shape):
    args = [torch.randn(M, D, dtype=torch.bfloat16, requires_grad=True),
            torch.randn(*w1_shape, dtype=torch.bfloat16, requires_grad=True),
            torch.randn(Dout, H, dtype=torch.bfloat16, requires_grad=True),
            torch.randn(M, Dout, dtype=torch.bfloat16)]

    def f(x, w1, w2, gy):
        y = fn(x, w1, w2)
        return (y,) + torch.autograd.grad(y, [x, w1, w2], gy)

    return make_fx(f, tracing_mode="fake")(*args)


def _targets(g):
    return [str(n.target) for n in g.graph.nodes if n.op == "call_function"]


@pytest.mark.parametrize("fn,w1_shape", [
    (SR.SwiGLUMemoryOptimizedFunction.apply, (2 * H, D)),
    (SR.SwiGLUFullCheckpointFunction.apply, (2 * H, D)),
], ids=["recompute", "full_checkpoint"])
@pytest.mark.parametrize("mode", ["emit_h", "prologue"])
def test_fwd_bwd_traces_through_registered_ops(traced, fn, w1_shape, mode):
    ops.set_dw2_mode(mode)
    g = _trace(fn, w1_shape)
    t = _targets(g)
    ours = [x for x in t if x.startswith("swiglu_b200.")]
    foreign = [x for x in t if not x.startswith("swiglu_b200.") and not x.startswith("aten.view")
               and not x.startswith("aten.empty") and not x.startswith("aten._unsafe_view")
               and x != "<built-in function getitem>"]
    assert not foreign, foreign                     # no aten matmul / pointwise fallbacks
    assert "swiglu_b200.bwd_grad_preact_.default" in ours
    assert ("swiglu_b200.bwd_dw2.default" in ours) == (mode == "prologue")
    assert sum(x == "swiglu_b200.matmul.default" for x in ours) == (4 if mode == "emit_h" else 3)
    outs = [n for n in g.graph.nodes if n.op == "output"][0].args[0]
    shapes = [tuple(o.meta["val"].shape) for o in outs]
    assert shapes == [(M, Dout), (M, D), w1_shape, (Dout, H)]


@pytest.mark.parametrize("fn", [FF.fused_matmul_swiglu_save_preact, FP.fused_swiglu_save_preact_packed,
                                FP.fused_swiglu_packed_no_save])
def test_fused_forward_entry_points_trace(traced, fn):
    """The fused modules' forward entry points assert CUDA inputs (as the
    reference does), so they are traced with fake CUDA tensors; their
    backward is the shared recompute backward traced above."""
    from torch._subclasses.fake_tensor import FakeTensorMode

    mode = FakeTensorMode()
    with mode:
        x = torch.empty(M, D, dtype=torch.bfloat16, device="cuda")
        w = torch.empty(D, 2 * H, dtype=torch.bfloat16, device="cuda")
        g = make_fx(lambda a, b: fn(a, b))(x, w)
    t = [x for x in _targets(g) if x != "<built-in function getitem>"]
    assert t and all(x.startswith("swiglu_b200.swiglu_fwd") for x in t), t


def test_inference_traces_h_only(traced):
    x = torch.randn(M, D, dtype=torch.bfloat16)
    w1 = torch.randn(2 * H, D, dtype=torch.bfloat16)
    w2 = torch.randn(Dout, H, dtype=torch.bfloat16)
    g = make_fx(lambda a, b, c: SR.SwiGLUMemoryOptimizedFunction.apply(a, b, c), tracing_mode="fake")(x, w1, w2)
    t = _targets(g)
    assert "swiglu_b200.swiglu_fwd_h.default" in t and "swiglu_b200.swiglu_fwd.default" not in t


@pytest.mark.parametrize("mode", ["emit_h", "prologue"])
def test_e4m3_forward_traces_through_registered_ops(traced, mode):
    """SwiGLUFP8ForwardFunction under tracing: four quantisations, the e4m3
    GEMM1 + SwiGLU and y GEMM, then the bf16 recompute backward, all as this
    library's registered ops."""
    ops.set_dw2_mode(mode)
    g = _trace(SR.SwiGLUFP8ForwardFunction.apply, (2 * H, D))
    t = _targets(g)
    ours = [x for x in t if x.startswith("swiglu_b200.")]
    assert sum(x == "swiglu_b200.quantize_e4m3.default" for x in ours) == 4
    assert "swiglu_b200.swiglu_fwd_e4m3.default" in ours and "swiglu_b200.matmul_e4m3.default" in ours
    assert "swiglu_b200.bwd_grad_preact_.default" in ours
    outs = [n for n in g.graph.nodes if n.op == "output"][0].args[0]
    assert [tuple(o.meta["val"].shape) for o in outs] == [(M, Dout), (M, D), (2 * H, D), (Dout, H)]


def test_mutation_is_declared():
    schema = torch.ops.swiglu_b200.bwd_grad_preact_.default._schema
    written = [a.name for a in schema.arguments if a.alias_info is not None and a.alias_info.is_write]
    assert written == ["preact", "h_out"]
    for name in ("swiglu_fwd", "swiglu_fwd_h", "swiglu_fwd_preact", "matmul", "bwd_dw2", "quantize_e4m3",
                 "swiglu_fwd_e4m3", "swiglu_fwd_e4m3_h", "matmul_e4m3"):
        s = getattr(torch.ops.swiglu_b200, name).default._schema
        assert not any(a.alias_info is not None and a.alias_info.is_write for a in s.arguments), name


def test_registered_op_has_no_cpu_kernel():
    a = torch.randn(16, 16, dtype=torch.bfloat16)
    with pytest.raises((NotImplementedError, RuntimeError)):
        torch.ops.swiglu_b200.matmul(a, a, False, False)
