"""Seeded synthetic inputs of the benchmark configurations.

x, grad_y ~ N(0, 1); W1 [2H, D], W2 [Dout, H] ~ N(0, fan_in^-1/2)
(fused_forward.py:359-360), drawn in f32 on the CPU in the order x, W1, W2,
grad_y and then cast, so every backend and every rank sees the same bits.
The test oracle draws its inputs the same way; tests check the two agree.
"""
from __future__ import annotations

import torch


def make_inputs(M: int, D: int, H: int, Dout: int, seed: int = 0, dtype=torch.float32):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(M, D, generator=g)
    w1 = torch.randn(2 * H, D, generator=g) * D ** -0.5
    w2 = torch.randn(Dout, H, generator=g) * H ** -0.5
    gy = torch.randn(M, Dout, generator=g)
    return tuple(t.to(dtype) for t in (x, w1, w2, gy))


def make_inputs_on_device(M: int, D: int, H: int, Dout: int, device, seed: int = 0,
                          dtype=torch.bfloat16):
    """The same distributions drawn by a generator on `device` (no host copy of
    the f32 draws, for shapes whose inputs are gigabytes). The bits differ from
    `make_inputs`; every rank that passes the same seed gets the same tensors."""
    g = torch.Generator(device=device).manual_seed(seed)
    out = []
    for shape, scale in (((M, D), 1.0), ((2 * H, D), D ** -0.5), ((Dout, H), H ** -0.5), ((M, Dout), 1.0)):
        t = torch.randn(*shape, generator=g, device=device)
        if scale != 1.0:
            t.mul_(scale)
        out.append(t.to(dtype))
        del t
    return tuple(out)
