"""Tensor-parallel block on 2+ GPUs (one process per GPU, NCCL).

GPU only; skipped unless at least two CUDA devices are visible. Each rank
runs the TP forward/backward on its token shard with its hidden-unit shard of
the weights; rank 0 gathers y, dx, dW1, dW2 and compares them with the oracle
on the full, unsharded problem (bounds as in test_gpu_parity.py).
"""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from oracle import swiglu_oracle as O

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, shape, fused, chunks, q):
    from datetime import timedelta

    import torch.distributed as dist
    from swiglu_b200 import tp

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=timedelta(seconds=60))
    try:
        M, D, H, Dout = shape
        x, w1, w2, gy = O.make_inputs(M, D, H, Dout, seed=11, dtype=torch.bfloat16)
        ms = M // world
        frs = None
        if fused:
            frs = tp.FusedReduceScatter()
            frs.K_PER_LINK_BYTE = 0          # always fuse at this small test shape
        mlp = tp.SwiGLUMLPTensorParallel(D, H, Dout, dtype=torch.bfloat16, fused_rs=frs if fused else False,
                                         chunks=chunks).to(dev).load_full(w1, w2)
        xl = x[rank * ms:(rank + 1) * ms].to(dev).requires_grad_(True)
        y = mlp(xl)
        dx, dw1, dw2 = torch.autograd.grad(y, [xl, mlp.w1, mlp.w2], gy[rank * ms:(rank + 1) * ms].to(dev))
        # a second step through the same buffers (epoch advance, buffer reuse)
        y2 = mlp(xl.detach().requires_grad_(True))
        assert torch.equal(y2.detach(), y.detach())
        outs = [y.detach(), dx, dw1, dw2]
        gathered = []
        for t in outs:
            buf = [torch.empty_like(t) for _ in range(world)]
            dist.all_gather(buf, t.contiguous())
            gathered.append([b.cpu() for b in buf])
        if rank == 0:
            q.put(gathered)
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("chunks", [1, 2], ids=["whole", "2_pieces"])
@pytest.mark.parametrize("fused", [True, False], ids=["fused_rs", "nccl_rs"])
@pytest.mark.parametrize("world", [2])
def test_tensor_parallel_matches_oracle(world, fused, chunks):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    from swiglu_b200 import tp

    shape = (512, 512, 1024, 384)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, shape, fused, chunks, q)) for r in range(world)]
    for p in procs:
        p.start()
    ys, dxs, dw1s, dw2s = q.get(timeout=300)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    M, D, H, Dout = shape
    x, w1, w2, gy = O.make_inputs(M, D, H, Dout, seed=11, dtype=torch.bfloat16)
    out = {"y": torch.cat(ys), "dx": torch.cat(dxs), "dw1": tp.unshard_w1_rows(dw1s),
           "dw2": torch.cat(dw2s, dim=1)}
    ref = O.mlp_forward_backward(x, w1, w2, gy, bf16=True)
    gt = O.ground_truth(x.float(), w1.float(), w2.float(), gy.float())
    for k in ("y", "dx", "dw1", "dw2"):
        assert O.rel_max(out[k], gt[k]) <= 7e-3, (k, O.rel_max(out[k], gt[k]))
        assert O.rel_max(out[k], ref[k]) <= 1e-2, (k, O.rel_max(out[k], ref[k]))
