"""Tensor-level wrappers over the C ABI.

Each function takes contiguous CUDA tensors, allocates its outputs through the
torch caching allocator (so `torch.cuda.max_memory_allocated` accounts for
them, as it does for the reference's `torch.empty` outputs,
fused_forward.py:216-217), makes the tensors' device current and enqueues the
native kernels on that device's current torch stream.
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib
from ._lib import BF16, F32, LAYOUT_PACKED128, LAYOUT_STD, W1_ROWS, W1_T  # noqa: F401

# Tile-order group (in 128-row tiles) where the caller passes none; the value
# the C side uses for the GEMMs it launches without one (kDefaultGroupM).
DEFAULT_GROUP_M = 32


def dtype_code(dtype: torch.dtype) -> int:
    if dtype == torch.bfloat16:
        return BF16
    if dtype == torch.float32:
        return F32
    raise TypeError(f"swiglu_b200 supports torch.bfloat16 and torch.float32, got {dtype}")


def _p(t: torch.Tensor | None) -> ctypes.c_void_p:
    return ctypes.c_void_p(0 if t is None else t.data_ptr())


# Stream-K workspace per (device index, stream handle): registered with the
# library the first time a stream is used, zero-filled by a memset ordered on
# that stream, and kept for the life of the process.
STREAM_WORKSPACE_BYTES = 48 << 20
_workspaces: dict[tuple[int, int], torch.Tensor] = {}
_stream_k = True


def _stream(dev: torch.device) -> ctypes.c_void_p:
    """Handle of `dev`'s current torch stream (the caller has made `dev`
    current), with its stream-K workspace registered."""
    s = torch.cuda.current_stream(dev).cuda_stream
    key = (dev.index, s)
    # No registration inside a graph capture: the buffer would belong to the
    # graph's private memory pool.
    if _stream_k and key not in _workspaces and not torch.cuda.is_current_stream_capturing():
        buf = torch.zeros(STREAM_WORKSPACE_BYTES, dtype=torch.uint8, device=dev)
        _lib.call("swiglu_b200_set_stream_workspace", _p(buf), buf.numel(), ctypes.c_void_p(s))
        _workspaces[key] = buf
    return ctypes.c_void_p(s)


# How the backward forms dW2 (read by the recompute Functions and the
# tensor-parallel block):
#   "prologue"  (default) dW2 recomputes h inside its operand prologue, before
#               the grad_h GEMM overwrites preact: no [M, H] buffer anywhere
#               in the backward (swiglu_recompute.py:71-73 without the h
#               temporary the reference materialises);
#   "emit_h"    the grad_h GEMM's epilogue also writes h of the preact it
#               replaces to a transient [M, H] buffer and dW2 = grad_y^T h is
#               a plain GEMM: faster by the difference of the two dW2 kernels
#               (about 0.26 ms of a 7.8 ms step at M=11136 D=3584 H=14336),
#               for one [M, H] buffer between the two GEMMs.
DW2_MODES = ("prologue", "emit_h")
_dw2_mode = "prologue"


def set_dw2_mode(mode: str) -> None:
    global _dw2_mode
    if mode not in DW2_MODES:
        raise ValueError(f"dW2 mode must be one of {DW2_MODES}, got {mode!r}")
    _dw2_mode = mode


def dw2_mode() -> str:
    return _dw2_mode


def set_stream_k(enabled: bool) -> None:
    """Enables (default) or disables the stream-K tail of the 2-SM GEMMs for
    later calls. Disabling unregisters every workspace this module registered;
    the kernels then run unsplit (results differ in f32 summation order)."""
    global _stream_k
    _stream_k = bool(enabled)
    if not enabled:
        for (index, s) in list(_workspaces):
            with torch.cuda.device(index):
                _lib.call("swiglu_b200_set_stream_workspace", None, 0, ctypes.c_void_p(s))
                torch.cuda.synchronize()
        _workspaces.clear()


# Launch trace: with a list installed by trace_launches(), every kernel entry
# point called through this module also records a CUDA event before and after
# its launch on the launching stream and appends (entry point, start, end).
# The events cost no device time worth measuring, so a caller (bench.py) can
# time each kernel inside the very steps it times as a whole.
_trace: list | None = None


def trace_launches(records: list | None) -> None:
    """Install `records` (a list) to collect (entry point, start event, end
    event) per launch from now on; None stops tracing."""
    global _trace
    _trace = records


def _call(dev: torch.device, name: str, *args) -> None:
    if _trace is None:
        _lib.call(name, *args)
        return
    st = torch.cuda.current_stream(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    _lib.call(name, *args)
    e1.record(st)
    _trace.append((name, e0, e1))


def _check_cuda(*ts: torch.Tensor) -> torch.device:
    dev = None
    for t in ts:
        if t is None:
            continue
        if not t.is_cuda:
            raise ValueError("swiglu_b200 kernels take CUDA tensors (there is no CPU path)")
        if not t.is_contiguous():
            raise ValueError("swiglu_b200 kernels take contiguous tensors")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise ValueError(f"tensors on different devices: {dev} vs {t.device}")
    return dev


def _same_dtype(*ts: torch.Tensor) -> torch.dtype:
    dt = None
    for t in ts:
        if t is None:
            continue
        if dt is None:
            dt = t.dtype
        elif t.dtype != dt:
            raise TypeError(f"mixed dtypes {dt} and {t.dtype}")
    return dt


def swiglu_fwd(x: torch.Tensor, w: torch.Tensor, *, w_form: int, layout: int,
               h_from_rounded: bool, want_h: bool = True, want_preact: bool = True,
               group_size_m: int = DEFAULT_GROUP_M, preact_out: torch.Tensor | None = None,
               h_out: torch.Tensor | None = None):
    """(preact [M, 2H] or None, h [M, H] or None) for preact = x . W1^T in one
    launch. want_preact=False is the no-save (inference) forward. preact_out /
    h_out: contiguous buffers to write into instead of new ones."""
    assert want_h or want_preact
    dev = _check_cuda(x, w, preact_out, h_out)
    dt = _same_dtype(x, w, preact_out, h_out)
    M, K = x.shape
    if w_form == W1_ROWS:
        n2, K2 = w.shape
    else:
        K2, n2 = w.shape
    assert K == K2 and n2 % 2 == 0, f"shape mismatch x{tuple(x.shape)} w{tuple(w.shape)}"
    H = n2 // 2
    if preact_out is not None:
        assert want_preact and preact_out.shape == (M, n2)
    if h_out is not None:
        assert want_h and h_out.shape == (M, H)
    preact = (preact_out if preact_out is not None else torch.empty((M, n2), device=dev, dtype=dt)) \
        if want_preact else None
    h = (h_out if h_out is not None else torch.empty((M, H), device=dev, dtype=dt)) if want_h else None
    with torch.cuda.device(dev):
        _call(dev, "swiglu_b200_fused_matmul_swiglu_save_preact", _p(x), _p(w), _p(preact), _p(h),
              M, K, H, dtype_code(dt), w_form, layout, int(bool(h_from_rounded)),
              int(group_size_m), _stream(dev))
    return preact, h


def matmul(a: torch.Tensor, b: torch.Tensor, *, a_t: bool, b_t: bool,
           out_dtype: torch.dtype | None = None, out: torch.Tensor | None = None,
           group_size_m: int = DEFAULT_GROUP_M, tile_n: int = 0) -> torch.Tensor:
    """C = op(a) . op(b); op(a) = a.T if a_t, op(b) = b.T if b_t. tile_n = 512
    asks the 2-SM kernel for 256 x 512 output tiles (long-K GEMMs), 256 for
    256 x 256; 0 chooses by size (512 from 8 waves of 256 x 512 tiles)."""
    dev = _check_cuda(a, b, out)
    dt = _same_dtype(a, b)
    M, K = (a.shape[1], a.shape[0]) if a_t else tuple(a.shape)
    Kb, N = (b.shape[1], b.shape[0]) if b_t else tuple(b.shape)
    assert K == Kb, f"inner dimensions differ: {K} vs {Kb}"
    odt = out_dtype or dt
    if out is None:
        out = torch.empty((M, N), device=dev, dtype=odt)
    else:
        assert out.shape == (M, N) and out.dtype == odt
    with torch.cuda.device(dev):
        _call(dev, "swiglu_b200_matmul_tiled", _p(a), _p(b), _p(out), M, N, K, int(a_t), int(b_t),
              dtype_code(dt), dtype_code(odt), int(group_size_m), int(tile_n), _stream(dev))
    return out


def bwd_dw2(grad_y: torch.Tensor, preact: torch.Tensor, *, layout: int,
            out: torch.Tensor | None = None) -> torch.Tensor:
    """dW2 [Dout, H] = grad_y^T . swiglu(preact), h recomputed in the GEMM prologue."""
    dev = _check_cuda(grad_y, preact, out)
    dt = _same_dtype(grad_y, preact)
    M, Dout = grad_y.shape
    M2, n2 = preact.shape
    assert M == M2 and n2 % 2 == 0
    H = n2 // 2
    if out is None:
        out = torch.empty((Dout, H), device=dev, dtype=dt)
    with torch.cuda.device(dev):
        _call(dev, "swiglu_b200_bwd_dw2", _p(grad_y), _p(preact), _p(out), M, H, Dout,
              dtype_code(dt), layout, _stream(dev))
    return out


def bwd_grad_preact_inplace(grad_y: torch.Tensor, w2: torch.Tensor, preact: torch.Tensor, *,
                            layout: int, h_out: torch.Tensor | None = None) -> torch.Tensor:
    """preact <- grad_preact, from grad_h = grad_y . W2 formed tile by tile (never stored).
    With `h_out` ([M, H]) the same epilogue also writes h = swiglu(preact) of
    the values it replaces."""
    dev = _check_cuda(grad_y, w2, preact, h_out)
    dt = _same_dtype(grad_y, w2, preact, h_out)
    M, Dout = grad_y.shape
    Dout2, H = w2.shape
    assert Dout == Dout2 and preact.shape == (M, 2 * H)
    with torch.cuda.device(dev):
        if h_out is None:
            _call(dev, "swiglu_b200_bwd_grad_preact_inplace", _p(grad_y), _p(w2), _p(preact), M, H, Dout,
                  dtype_code(dt), layout, _stream(dev))
        else:
            assert h_out.shape == (M, H)
            _call(dev, "swiglu_b200_bwd_grad_preact_inplace_emit_h", _p(grad_y), _p(w2), _p(preact),
                  _p(h_out), M, H, Dout, dtype_code(dt), layout, _stream(dev))
    return preact


def forward_logic(preact: torch.Tensor, *, layout: int) -> torch.Tensor:
    dev = _check_cuda(preact)
    M, n2 = preact.shape
    assert n2 % 2 == 0
    H = n2 // 2
    h = torch.empty((M, H), device=dev, dtype=preact.dtype)
    with torch.cuda.device(dev):
        _call(dev, "swiglu_b200_forward_logic", _p(preact), _p(h), M, H, dtype_code(preact.dtype),
              layout, _stream(dev))
    return h


def backward_logic(preact: torch.Tensor, grad_h: torch.Tensor, *, layout: int,
                   out: torch.Tensor | None = None) -> torch.Tensor:
    dev = _check_cuda(preact, grad_h, out)
    dt = _same_dtype(preact, grad_h)
    M, n2 = preact.shape
    H = n2 // 2
    assert grad_h.shape == (M, H), f"grad_h {tuple(grad_h.shape)} vs preact {tuple(preact.shape)}"
    if out is None:
        out = torch.empty_like(preact)
    with torch.cuda.device(dev):
        _call(dev, "swiglu_b200_backward_logic", _p(preact), _p(grad_h), _p(out), M, H, dtype_code(dt),
              layout, _stream(dev))
    return out


def pack_chunked(w: torch.Tensor, block_n_half: int, *, unpack: bool) -> torch.Tensor:
    dev = _check_cuda(w)
    K, n2 = w.shape
    out = torch.empty_like(w)
    with torch.cuda.device(dev):
        _call(dev, "swiglu_b200_pack_weight_chunked", _p(w), _p(out), K, n2 // 2, int(block_n_half),
              dtype_code(w.dtype), int(bool(unpack)), _stream(dev))
    return out


def device_status(device: torch.device | int | None = None, clear: bool = True) -> int:
    """Pipeline-timeout bits recorded by the kernels on `device` (0 = healthy)."""
    with torch.cuda.device(device if device is not None else torch.cuda.current_device()):
        return _lib.device_status(clear)


# ------------------------------------------------------------ e4m3 (FP8) path
def quantize_rows_e4m3(t: torch.Tensor):
    """(q, scale): row-scaled e4m3 copy of a bf16 [R, C] matrix, q [R, C]
    (torch.float8_e4m3fn) and the f32 dequantisation factor scale [R]
    (row r holds e4m3(v * 448 / amax_r), scale_r = amax_r / 448)."""
    dev = _check_cuda(t)
    if t.dtype != torch.bfloat16 or t.dim() != 2:
        raise TypeError("quantize_rows_e4m3 takes a 2-D bf16 tensor")
    R, C = t.shape
    q = torch.empty((R, C), device=dev, dtype=torch.float8_e4m3fn)
    s = torch.empty((R,), device=dev, dtype=torch.float32)
    with torch.cuda.device(dev):
        _call(dev, "swiglu_b200_quantize_rows_e4m3", _p(t), _p(q), _p(s), R, C, BF16, _stream(dev))
    return q, s


def swiglu_fwd_e4m3(xq: torch.Tensor, x_scale: torch.Tensor, wq: torch.Tensor, w_scale: torch.Tensor, *,
                    layout: int, h_from_rounded: bool, want_h: bool = True, want_preact: bool = True,
                    group_size_m: int = DEFAULT_GROUP_M):
    """(preact [M, 2H] or None, h [M, H] or None) in bf16 from e4m3 x [M, K]
    and W1 [2H, K] (rows in `layout` order) with their row scales."""
    assert want_h or want_preact
    dev = _check_cuda(xq, x_scale, wq, w_scale)
    M, K = xq.shape
    n2, K2 = wq.shape
    assert K == K2 and n2 % 2 == 0 and x_scale.shape == (M,) and w_scale.shape == (n2,)
    H = n2 // 2
    preact = torch.empty((M, n2), device=dev, dtype=torch.bfloat16) if want_preact else None
    h = torch.empty((M, H), device=dev, dtype=torch.bfloat16) if want_h else None
    with torch.cuda.device(dev):
        _call(dev, "swiglu_b200_fused_matmul_swiglu_e4m3", _p(xq), _p(x_scale), _p(wq), _p(w_scale),
              _p(preact), _p(h), M, K, H, layout, int(bool(h_from_rounded)), int(group_size_m), _stream(dev))
    return preact, h


def matmul_e4m3(aq: torch.Tensor, a_scale: torch.Tensor, bq: torch.Tensor, b_scale: torch.Tensor, *,
                out_dtype: torch.dtype = torch.bfloat16, group_size_m: int = DEFAULT_GROUP_M) -> torch.Tensor:
    """C [M, N] = A . B^T for e4m3 A [M, K] and B [N, K] with their row scales."""
    dev = _check_cuda(aq, a_scale, bq, b_scale)
    M, K = aq.shape
    N, K2 = bq.shape
    assert K == K2 and a_scale.shape == (M,) and b_scale.shape == (N,)
    out = torch.empty((M, N), device=dev, dtype=out_dtype)
    with torch.cuda.device(dev):
        _call(dev, "swiglu_b200_matmul_e4m3", _p(aq), _p(a_scale), _p(bq), _p(b_scale), _p(out), M, N, K,
              dtype_code(out_dtype), int(group_size_m), _stream(dev))
    return out
