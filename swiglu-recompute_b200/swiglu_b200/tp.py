"""Tensor-parallel SwiGLU MLP block (Megatron column -> row split, sequence-
parallel edges) over torch.distributed; NCCL over NVLink on B200.

Rank r of t owns hidden units [r*H/t, (r+1)*H/t):
  W1 shard  [2H/t, D]  = the left rows AND the gate rows of those units
                         (left/gate pairs stay on one rank, so SwiGLU is local)
  W2 shard  [Dout, H/t] = the matching columns of W2
Tokens are sharded along M: each rank holds x_r [M/t, D] and y_r [M/t, Dout].

forward   x = all_gather(x_r) ; preact_r, h_r = GEMM1+SwiGLU(x, W1_r)
          y_partial = h_r . W2_r^T (f32) ; y_r = reduce_scatter(y_partial)
backward  grad_y = all_gather(grad_y_r)
          preact_r <- grad_preact_r (in place) ; dW1_r = grad_preact_r^T . x
          dW2_r = grad_y^T . h_r, h_r recomputed from preact_r as the
          single-GPU backward does (ops.dw2_mode: inside the dW2 kernel's
          operand prologue, or written by the grad_preact epilogue)
          dx_partial = grad_preact_r . W1_r (f32) ; dx_r = reduce_scatter(dx_partial)
Partials are reduced in f32 and rounded once, so the result does not depend
on how many bf16 hops a ring reduction takes.

The reference is single-GPU only; this layer adds the multi-GPU path of the
benchmark's tensor-parallel configuration (same math per rank as
SwiGLUMemoryOptimizedFunction, swiglu_recompute.py:58-78).
"""
from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist
import torch.nn as nn

from . import ops
from .ops import LAYOUT_PACKED128, LAYOUT_STD, W1_ROWS


# ------------------------------------------------------------- sharding
def shard_w1_rows(w1: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    """Rows of W1 [2H, D] (standard [left; gate]) owned by `rank`: [2H/t, D]."""
    H = w1.shape[0] // 2
    assert H % world == 0, f"H={H} must divide evenly over {world} ranks"
    hs = H // world
    lo, hi = rank * hs, (rank + 1) * hs
    return torch.cat([w1[lo:hi], w1[H + lo:H + hi]], dim=0).contiguous()


def shard_w2(w2: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    """Columns of W2 [Dout, H] owned by `rank`: [Dout, H/t]."""
    H = w2.shape[1]
    assert H % world == 0
    hs = H // world
    return w2[:, rank * hs:(rank + 1) * hs].contiguous()


def unshard_w1_rows(shards: list[torch.Tensor]) -> torch.Tensor:
    """Inverse of shard_w1_rows over all ranks' shards."""
    hs = shards[0].shape[0] // 2
    return torch.cat([s[:hs] for s in shards] + [s[hs:] for s in shards], dim=0)


# ---------------------------------------------------------- collectives
def all_gather_rows(t: torch.Tensor, group=None) -> torch.Tensor:
    world = dist.get_world_size(group)
    out = torch.empty((t.shape[0] * world, *t.shape[1:]), dtype=t.dtype, device=t.device)
    dist.all_gather_into_tensor(out, t.contiguous(), group=group)
    return out


def reduce_scatter_rows(t: torch.Tensor, group=None) -> torch.Tensor:
    world = dist.get_world_size(group)
    assert t.shape[0] % world == 0
    out = torch.empty((t.shape[0] // world, *t.shape[1:]), dtype=t.dtype, device=t.device)
    dist.reduce_scatter_tensor(out, t.contiguous(), group=group)
    return out


class _PendingReduceScatter:
    """An NCCL reduce-scatter in flight on the collective's own stream; the
    input stays referenced until `wait` joins the result into the current stream."""

    def __init__(self, t: torch.Tensor, group=None):
        world = dist.get_world_size(group)
        assert t.shape[0] % world == 0
        self.inp = t.contiguous()
        self.out = torch.empty((t.shape[0] // world, *t.shape[1:]), dtype=t.dtype, device=t.device)
        self.work = dist.reduce_scatter_tensor(self.out, self.inp, group=group, async_op=True)

    def wait(self) -> torch.Tensor:
        self.work.wait()
        self.inp = None
        return self.out


# ------------------------------------------- fused GEMM -> reduce-scatter
class FusedReduceScatter:
    """Receive buffers in symmetric (peer-mapped) memory for the reduce-scatter
    of an f32 partial product, fused into the producing GEMM.

    For a partial D [M, N] on every rank (M = world * rows_per_rank), the GEMM
    epilogue stores row r into rank r // rows_per_rank's receive buffer
    [world, rows_per_rank, N] at slot [this rank, r % rows_per_rank] over
    NVLink while the other tiles are still computing; a signal kernel then
    publishes the call's epoch into every owner's flag slot for this rank, and
    each owner sums its `world` slots in fixed rank order (deterministic) and
    rounds once. Buffers are reused across calls: between two uses of the
    same buffer every rank passes through other collectives of the step, which
    orders the next writes after the previous reduction.
    """

    def __init__(self, group=None, fuse=("y", "dx")):
        # `fuse`: the reduce-scatters (of "y", "dx") that may ride on their
        # GEMM; each still only where wants() finds its math covers its push,
        # except those named in `always` (set by the caller after construction).
        self.fuse = tuple(fuse)
        self.always = ()
        self.group = group if group is not None else dist.group.WORLD
        self.world = dist.get_world_size(self.group)
        self.rank = dist.get_rank(self.group)
        self.epoch = 0
        self._slots = {}

    def _slot(self, key, rows_per_rank, n, device):
        k = (key, rows_per_rank, n)
        if k not in self._slots:
            import torch.distributed._symmetric_memory as symm_mem
            recv = symm_mem.empty(self.world * rows_per_rank * n, dtype=torch.float32, device=device)
            recv_h = symm_mem.rendezvous(recv, self.group)
            flags = symm_mem.empty(self.world, dtype=torch.int32, device=device)
            flags.zero_()
            flags_h = symm_mem.rendezvous(flags, self.group)
            torch.cuda.synchronize(device)
            dist.barrier(group=self.group)
            peers = (ctypes.c_void_p * self.world)(*[recv_h.buffer_ptrs[i] for i in range(self.world)])
            peer_flags = (ctypes.c_void_p * self.world)(*[flags_h.buffer_ptrs[i] for i in range(self.world)])
            self._slots[k] = (recv, recv_h, flags, flags_h, peers, peer_flags)
        return self._slots[k]

    # Fused only when the GEMM's math covers its NVLink push: per rank the
    # GEMM takes ~2MNK / 1.3 PFLOP/s while (world-1)/world of its 4MN bytes
    # leave at ~0.6 TB/s, i.e. K >= 4333 (world-1) / world. Measured at
    # config 2 (M=11136): world 2 fused 4.60 ms/step vs NCCL 4.96; world 8
    # (y: K=1792, dx: K=3584) fused 2.18 vs NCCL 2.05 (before the backward
    # deferred dx's reduction behind dW2/dW1; after it 2.03 vs 1.85).
    K_PER_LINK_BYTE = 4333

    def wants(self, k, which="y"):
        """Whether the scatter GEMM with inner dimension k should carry the
        reduce-scatter of `which` ("y" or "dx"): its math covers its NVLink
        push, or `which` is in `always`. Measured with dx deferred behind
        dW2/dW1 at world 8 (dx K=3584, below the line): fused 2.03 ms/step vs
        NCCL 1.85, so the rule holds there too."""
        if which not in self.fuse:
            return False
        return which in self.always or k * self.world >= self.K_PER_LINK_BYTE * (self.world - 1)

    def matmul_start(self, key, a, b, *, a_t, b_t, out_dtype):
        """Enqueues the scatter GEMM of op(a) . op(b) and its signal; returns a
        pending handle for `finish`. Work enqueued in between overlaps the
        other ranks' pushes into this rank's receive buffer."""
        from ._lib import BF16
        from .ops import _call, _p, _stream

        M = a.shape[1] if a_t else a.shape[0]
        K = a.shape[0] if a_t else a.shape[1]
        N = b.shape[0] if b_t else b.shape[1]
        assert M % self.world == 0
        rows = M // self.world
        dev = a.device
        recv, _, flags, _, peers, peer_flags = self._slot(key, rows, N, dev)
        self.epoch = (self.epoch + 1) & 0x7FFFFFFF or 1
        st = _stream(dev)
        with torch.cuda.device(dev):
            _call(dev, "swiglu_b200_matmul_scatter_rows", _p(a), _p(b), M, N, K, int(a_t), int(b_t), BF16,
                  peers, self.world, self.rank, rows, st)
            _call(dev, "swiglu_b200_tp_signal", peer_flags, self.world, self.rank, self.epoch, st)
        return (recv, flags, self.epoch, rows, N, out_dtype, dev)

    def finish(self, pending):
        """This rank's [M / world, N] rows: the owner's fixed-order sum of the
        `world` partials, once every rank's signal has arrived."""
        from .ops import _call, _p, _stream, dtype_code

        recv, flags, epoch, rows, N, out_dtype, dev = pending
        out = torch.empty((rows, N), device=dev, dtype=out_dtype)
        with torch.cuda.device(dev):
            _call(dev, "swiglu_b200_tp_reduce_rows", _p(recv), _p(flags), self.world, epoch, _p(out), rows, N,
                  dtype_code(out_dtype), _stream(dev))
        return out

    def matmul(self, key, a, b, *, a_t, b_t, out_dtype):
        """Reduce-scattered op(a) . op(b): returns this rank's [M / world, N] rows."""
        return self.finish(self.matmul_start(key, a, b, a_t=a_t, b_t=b_t, out_dtype=out_dtype))


# -------------------------------------------------------- local compute
class NativeCompute:
    """Per-rank compute on libswiglu_b200.so (bf16 tcgen05 or f32 kernels)."""

    @staticmethod
    def swiglu_fwd(x, w1_local, out=None):
        preact_out, h_out = out if out is not None else (None, None)
        return ops.swiglu_fwd(x, w1_local, w_form=W1_ROWS, layout=LAYOUT_STD, h_from_rounded=True,
                              preact_out=preact_out, h_out=h_out)

    @staticmethod
    def matmul(a, b, *, a_t, b_t, out_dtype=None, tile_n=0):
        return ops.matmul(a, b, a_t=a_t, b_t=b_t, out_dtype=out_dtype, tile_n=tile_n)

    @staticmethod
    def dw2(gy, preact):
        return ops.bwd_dw2(gy, preact, layout=LAYOUT_STD)

    @staticmethod
    def grad_preact_inplace(gy, w2_local, preact, h_out=None):
        return ops.bwd_grad_preact_inplace(gy, w2_local, preact, layout=LAYOUT_STD, h_out=h_out)


def _all_gather_chunks(t_local, group, chunks):
    """All-gather the row shard t_local [m, ...] as `chunks` row pieces, each an
    asynchronous NCCL all-gather into its slice of one buffer: rows
    [c*t*mc, (c+1)*t*mc) hold every rank's piece c (mc = m / chunks), rank by
    rank. Returns (buffer, works); work c must be waited on (which orders the
    current stream after it) before slice c is read."""
    world = dist.get_world_size(group)
    m = t_local.shape[0]
    mc = m // chunks
    out = torch.empty((m * world, *t_local.shape[1:]), dtype=t_local.dtype, device=t_local.device)
    works = []
    for c in range(chunks):
        piece = t_local[c * mc:(c + 1) * mc].contiguous()
        works.append(dist.all_gather_into_tensor(out[c * world * mc:(c + 1) * world * mc], piece, group=group,
                                                 async_op=True))
    return out, works


def tp_dw2_form(hidden_local: int, dout: int, pairs: int | None) -> str:
    """The dW2 form a rank's backward takes: the process-wide ops.dw2_mode(),
    except that the prologue kernel is replaced by the emit-h form when its
    launch would be shorter than two waves of its 256 x 512 pair tiles (the
    stream-K tail cannot fill a launch that short). Measured on 8 B200s at
    config 2 (10 steps, max over ranks): 8 ranks (H/t = 1792: 49 tiles for 74
    CTA pairs) prologue 2.037 ms/step vs emit-h 1.842; 4 ranks (98 tiles)
    2.737 vs 2.629; 2 ranks (196 tiles) equal. `pairs`: CTA pairs of the
    device (None: no native kernels, the process-wide mode)."""
    mode = ops.dw2_mode()
    if mode != "prologue" or pairs is None:
        return mode
    tiles = -(-hidden_local // 256) * -(-dout // 512)
    return "emit_h" if tiles < 2 * pairs else mode


def _pairs(device) -> int | None:
    if device.type != "cuda":
        return None
    return torch.cuda.get_device_properties(device).multi_processor_count // 2


class _TPSwiGLUFunction(torch.autograd.Function):
    """The tensor-parallel block. With `chunks` = C > 1 each rank's token
    shard travels as C row pieces: the all-gathers of x and grad_y are issued
    for all pieces at once, and the GEMMs of piece c start as soon as piece c
    has arrived while the later pieces are still in flight; y and grad_x are
    reduce-scattered piece by piece (the reduce-scatter of piece c overlaps
    the GEMMs of piece c + 1). Gathered rows are stored piece-major, which
    every GEMM of the block is indifferent to (dW1 and dW2 sum over all rows
    of both of their operands in the same order)."""

    @staticmethod
    def forward(ctx, x_local, w1_local, w2_local, group, compute, reduce_f32, fused_rs, chunks=1):
        world = dist.get_world_size(group)
        if chunks < 1 or x_local.shape[0] % chunks:
            chunks = 1
        x, works = _all_gather_chunks(x_local, group, chunks)
        rows = x.shape[0] // chunks
        n2 = w1_local.shape[0]
        preact = x.new_empty((x.shape[0], n2))
        h = x.new_empty((x.shape[0], n2 // 2))
        fused = fused_rs is not None and fused_rs.wants(h.shape[1], "y")
        acc_dt = torch.float32 if reduce_f32 else x.dtype
        pending = []
        for c in range(chunks):
            works[c].wait()
            sl = slice(c * rows, (c + 1) * rows)
            compute.swiglu_fwd(x[sl], w1_local, out=(preact[sl], h[sl]))
            if fused:
                pending.append(fused_rs.matmul_start(("y", c), h[sl], w2_local, a_t=False, b_t=True,
                                                     out_dtype=x.dtype))
            else:
                y_part = compute.matmul(h[sl], w2_local, a_t=False, b_t=True, out_dtype=acc_dt)
                pending.append(_PendingReduceScatter(y_part, group))
        del h
        pieces = [fused_rs.finish(p) if fused else p.wait().to(x.dtype) for p in pending]
        y_local = pieces[0] if chunks == 1 else torch.cat(pieces)
        ctx.save_for_backward(x, w1_local, w2_local, preact)
        ctx.group, ctx.compute, ctx.reduce_f32, ctx.fused_rs = group, compute, reduce_f32, fused_rs
        ctx.chunks, ctx.world = chunks, world
        return y_local

    @staticmethod
    def backward(ctx, grad_y_local):
        if getattr(ctx, "_consumed", False):
            raise RuntimeError("tensor-parallel SwiGLU backward already consumed its saved preact")
        ctx._consumed = True
        x, w1_local, w2_local, preact = ctx.saved_tensors
        compute, chunks = ctx.compute, ctx.chunks
        gy, works = _all_gather_chunks(grad_y_local.to(x.dtype).contiguous(), ctx.group, chunks)
        rows = gy.shape[0] // chunks
        emit = tp_dw2_form(preact.shape[1] // 2, w2_local.shape[0], _pairs(preact.device)) == "emit_h"
        # dW2 as in the single-GPU backward (tp_dw2_form): in the prologue
        # form the dW2 kernel reads every row of preact (and so of grad_y)
        # before grad_h replaces any of it; with emit_h the grad_h epilogue
        # writes h piece by piece and dW2 runs after the last piece.
        if not emit:
            for w in works:
                w.wait()
            dw2 = compute.dw2(gy, preact)
        h = torch.empty((preact.shape[0], preact.shape[1] // 2), device=preact.device,
                        dtype=preact.dtype) if emit else None
        fused = ctx.fused_rs is not None and ctx.fused_rs.wants(preact.shape[1], "dx")
        acc_dt = torch.float32 if ctx.reduce_f32 else x.dtype
        pending = []
        for c in range(chunks):
            works[c].wait()
            sl = slice(c * rows, (c + 1) * rows)
            gp = compute.grad_preact_inplace(gy[sl], w2_local, preact[sl], h_out=h[sl] if emit else None)
            # dx of this piece first: its reduce-scatter proceeds while the
            # later pieces, dW2 and dW1 (no communication) compute.
            if fused:
                pending.append(ctx.fused_rs.matmul_start(("dx", c), gp, w1_local, a_t=False, b_t=False,
                                                         out_dtype=x.dtype))
            else:
                pending.append(_PendingReduceScatter(
                    compute.matmul(gp, w1_local, a_t=False, b_t=False, out_dtype=acc_dt), ctx.group))
        torch.autograd.graph.increment_version(preact)
        gp = preact                                                  # now holds grad_preact
        if emit:
            dw2 = compute.matmul(gy, h, a_t=True, b_t=False)
            del h
        # Tile widths of the local GEMMs by size (256 x 512 from 8 waves of
        # them): the per-rank dW1 of a sharded block is 1/t of the
        # single-GPU one, often below the size where the wide tiles win.
        dw1 = compute.matmul(gp, x, a_t=True, b_t=False)
        pieces = [ctx.fused_rs.finish(p) if fused else p.wait().to(x.dtype) for p in pending]
        dx_local = pieces[0] if chunks == 1 else torch.cat(pieces)
        return dx_local, dw1, dw2, None, None, None, None, None


def tp_swiglu(x_local, w1_local, w2_local, group=None, compute=NativeCompute, reduce_f32=True, fused_rs=None,
              chunks=1):
    """y_r [M/t, Dout] for the token shard x_r [M/t, D]; see the module docstring.
    With `fused_rs` (a FusedReduceScatter) the reduce-scatters of y and grad_x
    run inside their GEMMs over NVLink instead of as NCCL collectives; with
    `chunks` > 1 the shard's collectives travel in that many row pieces,
    overlapped with the GEMMs of the pieces already there."""
    return _TPSwiGLUFunction.apply(x_local, w1_local, w2_local, group, compute, reduce_f32, fused_rs, chunks)


class SwiGLUMLPTensorParallel(nn.Module):
    """One SwiGLU MLP block split over the ranks of `group` (weights are this
    rank's shards: w1 [2H/t, D], w2 [Dout, H/t])."""

    def __init__(self, dim, hidden_dim, out_dim=None, dtype=torch.float32, group=None,
                 reduce_f32=True, fused_rs=None, chunks=1):
        super().__init__()
        self.group = group
        # Row pieces the token shard's collectives travel in (tp_swiglu).
        self.chunks = chunks
        # Fused GEMM + reduce-scatter over NVLink (bf16 only); default on for
        # bf16 when CUDA peer memory is available.
        self.fused_rs = fused_rs
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        assert hidden_dim % self.world == 0
        self.dim, self.hidden_dim = dim, hidden_dim
        self.out_dim = out_dim if out_dim is not None else dim
        self.reduce_f32 = reduce_f32
        hs = hidden_dim // self.world
        self.w1 = nn.Parameter(torch.empty(2 * hs, dim, dtype=dtype))
        self.w2 = nn.Parameter(torch.empty(self.out_dim, hs, dtype=dtype))

    @torch.no_grad()
    def load_full(self, w1: torch.Tensor, w2: torch.Tensor):
        self.w1.copy_(shard_w1_rows(w1, self.rank, self.world))
        self.w2.copy_(shard_w2(w2, self.rank, self.world))
        return self

    def forward(self, x_local):
        frs = None
        if self.fused_rs is not False and x_local.dtype == torch.bfloat16 and x_local.is_cuda:
            if self.fused_rs is None or self.fused_rs is True:
                self.fused_rs = FusedReduceScatter(self.group)
            frs = self.fused_rs
        return tp_swiglu(x_local, self.w1, self.w2, self.group, NativeCompute, self.reduce_f32, frs,
                         self.chunks)
