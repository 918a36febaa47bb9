"""Tensor-parallel host logic on CPU: sharding, all-gather / reduce-scatter
placement and the backward order, run as world_size-2 gloo ranks with the
oracle's math standing in for the per-rank CUDA kernels. CPU only."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import swiglu_oracle as O
from swiglu_b200 import tp


class OracleCompute:
    """Per-rank compute with the oracle's f32 math (test stand-in for NativeCompute)."""

    @staticmethod
    def swiglu_fwd(x, w1_local, out=None):
        preact = x @ w1_local.t()
        h = O.forward_logic(preact)
        if out is not None:
            out[0].copy_(preact)
            out[1].copy_(h)
            return out
        return preact, h

    @staticmethod
    def matmul(a, b, *, a_t, b_t, out_dtype=None, tile_n=0):
        out = (a.t() if a_t else a) @ (b.t() if b_t else b)
        return out.to(out_dtype) if out_dtype is not None else out

    @staticmethod
    def dw2(gy, preact):
        return gy.t() @ O.forward_logic(preact)

    @staticmethod
    def grad_preact_inplace(gy, w2_local, preact, h_out=None):
        if h_out is not None:
            h_out.copy_(O.forward_logic(preact))
        preact.copy_(O.backward_logic(preact, gy @ w2_local))
        return preact


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, M, D, H, Dout, q, dw2_mode="emit_h", chunks=1):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from swiglu_b200 import ops
        ops.set_dw2_mode(dw2_mode)
        torch.set_num_threads(1)
        x, w1, w2, gy = O.make_inputs(M, D, H, Dout, seed=3)
        ms = M // world
        w1_l = tp.shard_w1_rows(w1, rank, world).requires_grad_(True)
        w2_l = tp.shard_w2(w2, rank, world).requires_grad_(True)
        x_l = x[rank * ms:(rank + 1) * ms].clone().requires_grad_(True)
        y_l = tp.tp_swiglu(x_l, w1_l, w2_l, None, OracleCompute, True, None, chunks)
        dx_l, dw1_l, dw2_l = torch.autograd.grad(y_l, [x_l, w1_l, w2_l], gy[rank * ms:(rank + 1) * ms])
        q.put((rank, y_l.detach(), dx_l, dw1_l, dw2_l))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2])
@pytest.mark.parametrize("dw2_mode", ["emit_h", "prologue"])
@pytest.mark.parametrize("chunks", [1, 2, 4])
def test_tp_matches_single_rank_oracle(world, dw2_mode, chunks):
    """The block split over two gloo ranks, its collectives in `chunks` row
    pieces (piece-major gathered rows), against the unsplit oracle."""
    M, D, H, Dout = 64, 48, 128, 40
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, M, D, H, Dout, q, dw2_mode, chunks))
             for r in range(world)]
    for p in procs:
        p.start()
    res = sorted([q.get(timeout=120) for _ in range(world)], key=lambda t: t[0])
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    x, w1, w2, gy = O.make_inputs(M, D, H, Dout, seed=3)
    ref = O.mlp_forward_backward(x, w1, w2, gy)
    y = torch.cat([r[1] for r in res])
    dx = torch.cat([r[2] for r in res])
    dw1 = tp.unshard_w1_rows([r[3] for r in res])
    dw2 = torch.cat([r[4] for r in res], dim=1)
    assert O.rel_max(y, ref["y"]) <= 1e-5
    assert O.rel_max(dx, ref["dx"]) <= 1e-5
    assert O.rel_max(dw1, ref["dw1"]) <= 1e-5
    assert O.rel_max(dw2, ref["dw2"]) <= 1e-5


def test_shard_roundtrip():
    w1 = torch.randn(2 * 256, 32)
    shards = [tp.shard_w1_rows(w1, r, 4) for r in range(4)]
    assert all(s.shape == (128, 32) for s in shards)
    assert torch.equal(tp.unshard_w1_rows(shards), w1)
    # each shard holds left AND gate rows of the same hidden units
    assert torch.equal(shards[1][:64], w1[64:128])
    assert torch.equal(shards[1][64:], w1[256 + 64:256 + 128])
    w2 = torch.randn(16, 256)
    assert torch.equal(torch.cat([tp.shard_w2(w2, r, 4) for r in range(4)], dim=1), w2)


def _dying_worker(rank, world, port, q):
    from datetime import timedelta
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=5))
    if rank == 1:
        os._exit(3)          # a rank that dies between steps
    try:
        t = torch.ones(4, 2)
        tp.all_gather_rows(t)
        q.put("no error")
    except Exception as e:   # the survivor sees an error, not a hang
        q.put(type(e).__name__)


def test_dead_rank_surfaces_as_error():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_dying_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    msg = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert msg != "no error"


@pytest.mark.parametrize("world,H,y_fused,dx_fused", [
    (2, 14336, True, True),      # config 2: the GEMMs' math covers their NVLink push
    (4, 14336, True, True),
    (8, 14336, False, False),    # config 2 at 8 ranks: K = 1792 / 3584, NCCL measured faster
    (8, 28672, False, True),     # config 5 at 8 ranks: y K = 3584 stays on NCCL, dx K = 7168 fuses
])
def test_fused_reduce_scatter_crossover(world, H, y_fused, dx_fused):
    """The per-GEMM choice between the GEMM-fused reduce-scatter and NCCL:
    fused once K >= 4333 (t - 1) / t (y: K = H / t, dx: K = 2H / t)."""
    class Rule(tp.FusedReduceScatter):
        def __init__(self, w):  # the rule only, no process group
            self.world = w
            self.fuse, self.always = ("y", "dx"), ()

    r = Rule(world)
    assert r.wants(H // world, "y") == y_fused
    assert r.wants(2 * H // world, "dx") == dx_fused
    r.always = ("y",)                  # y fused at any size, dx still by the rule
    assert r.wants(H // world, "y") and r.wants(2 * H // world, "dx") == dx_fused
    r.fuse = ("dx",)                   # y never fused
    assert not r.wants(H // world, "y") and r.wants(2 * H // world, "dx") == dx_fused


def test_tp_dw2_form_rule():
    """The per-rank dW2 form: the prologue kernel where its launch has at
    least two waves of 256 x 512 pair tiles, the emit-h form below that."""
    from swiglu_b200 import ops
    prev = ops.dw2_mode()
    try:
        ops.set_dw2_mode("prologue")
        pairs = 74                                         # a B200: 148 SMs
        assert tp.tp_dw2_form(14336 // 2, 3584, pairs) == "prologue"   # config 2, 2 ranks: 196 tiles
        assert tp.tp_dw2_form(14336 // 4, 3584, pairs) == "emit_h"     # 98 tiles
        assert tp.tp_dw2_form(14336 // 8, 3584, pairs) == "emit_h"     # 49 tiles
        assert tp.tp_dw2_form(28672 // 8, 8192, pairs) == "prologue"   # config 5, 8 ranks: 224 tiles
        assert tp.tp_dw2_form(64, 40, None) == "prologue"              # no native kernels: as set
        ops.set_dw2_mode("emit_h")
        assert tp.tp_dw2_form(14336 // 2, 3584, pairs) == "emit_h"
    finally:
        ops.set_dw2_mode(prev)
