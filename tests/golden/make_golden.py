"""Generate the golden vectors in this directory by running the REFERENCE code.

    python tests/golden/make_golden.py --reference <path to tongzhou8086/swiglu-recompute>

Imports the reference's own modules (swiglu_recompute, fused_forward_packed)
on the CPU and records their outputs on small seeded inputs, so the CPU oracle
(oracle/swiglu_oracle.py) can be pinned against the reference without the
reference being present later (tests/test_oracle_golden.py reads only the
.npz files written here).

The reference's pointwise helpers are @torch.compile'd; Inductor's CPU backend
needs a working C++ compiler (CXX). With --eager, TORCHDYNAMO_DISABLE=1 runs
them eagerly instead (identical f32 results; bf16 then rounds per op).

Fixtures (all arrays float32; bf16 tensors hold exactly-representable values):
  mlp_f32.npz       recompute fwd+bwd, f32, M=64 D=64 H=128 Dout=64, plus GT
  mlp_bf16.npz      recompute fwd+bwd, bf16, same shape, plus GT (bf16)
  mlp_ragged.npz    recompute fwd+bwd, f32, M=40 D=24 H=136 Dout=16
  pointwise.npz     _swiglu_forward_logic / _swiglu_backward_logic (f32, M=8 H=256),
                    pack/unpack of a [4, 512] weight, _h_from_packed_preact
"""
from __future__ import annotations

import argparse
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def _np(t):
    return t.detach().float().cpu().numpy()


def _inputs(torch, M, D, H, Dout, seed, dtype):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(M, D, generator=g)
    w1 = torch.randn(2 * H, D, generator=g) * D ** -0.5
    w2 = torch.randn(Dout, H, generator=g) * H ** -0.5
    gy = torch.randn(M, Dout, generator=g)
    return [t.to(dtype) for t in (x, w1, w2, gy)]


def _mlp_case(torch, ref, M, D, H, Dout, seed, dtype):
    x, w1, w2, gy = _inputs(torch, M, D, H, Dout, seed, dtype)
    out = {"x": _np(x), "w1": _np(w1), "w2": _np(w2), "gy": _np(gy)}
    # Recompute Function through the reference's public module.
    rc = ref.SwiGLUMLPCustom(D, H, Dout, dtype=dtype)
    gt = ref.SwiGLUMLPGroundTruth(D, H, Dout, dtype=dtype)
    with torch.no_grad():
        for m in (rc, gt):
            m.w1.copy_(w1)
            m.w2.copy_(w2)
    for name, m in (("rc", rc), ("gt", gt)):
        xi = x.detach().clone().requires_grad_(True)
        y = m(xi)
        dx, dw1, dw2 = torch.autograd.grad(y, [xi, m.w1, m.w2], gy)
        out.update({f"{name}_y": _np(y), f"{name}_dx": _np(dx), f"{name}_dw1": _np(dw1),
                    f"{name}_dw2": _np(dw2)})
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    ap.add_argument("--eager", action="store_true")
    args = ap.parse_args()
    if args.eager:
        os.environ["TORCHDYNAMO_DISABLE"] = "1"
    sys.path.insert(0, os.path.abspath(args.reference))
    import torch
    import swiglu_recompute as ref
    import fused_forward_packed as refp

    torch.set_num_threads(min(8, os.cpu_count() or 1))
    meta = {"torch": torch.__version__, "eager": int(args.eager)}

    np.savez_compressed(os.path.join(HERE, "mlp_f32.npz"),
                        **_mlp_case(torch, ref, 64, 64, 128, 64, 0, torch.float32), **meta)
    np.savez_compressed(os.path.join(HERE, "mlp_bf16.npz"),
                        **_mlp_case(torch, ref, 64, 64, 128, 64, 1, torch.bfloat16), **meta)
    np.savez_compressed(os.path.join(HERE, "mlp_ragged.npz"),
                        **_mlp_case(torch, ref, 40, 24, 136, 16, 2, torch.float32), **meta)

    g = torch.Generator().manual_seed(3)
    M, H = 8, 256
    preact = torch.randn(M, 2 * H, generator=g)
    grad_h = torch.randn(M, H, generator=g)
    h = ref._swiglu_forward_logic(preact)
    gp = ref._swiglu_backward_logic(preact, grad_h)
    w = torch.arange(4 * 512, dtype=torch.float32).reshape(4, 512)
    packed = refp.pack_swiglu_weight_chunked_torch(w)
    packed64 = refp.pack_swiglu_weight_chunked_torch(w, block_n_half=64)
    unpacked = refp.unpack_swiglu_weight_chunked_torch(packed)
    lin = torch.arange(512 * 4, dtype=torch.float32).reshape(512, 4)
    lin_packed = refp.pack_swiglu_linear_weight(lin)
    ppre = refp.pack_swiglu_weight_chunked_torch(preact.contiguous())
    h_packed = refp._h_from_packed_preact(ppre, M, H // 128, 128)
    np.savez_compressed(os.path.join(HERE, "pointwise.npz"), preact=_np(preact), grad_h=_np(grad_h),
                        h=_np(h), grad_preact=_np(gp), w=_np(w), packed=_np(packed),
                        packed64=_np(packed64), unpacked=_np(unpacked), lin=_np(lin),
                        lin_packed=_np(lin_packed), preact_packed=_np(ppre), h_packed=_np(h_packed),
                        **meta)
    print("wrote", sorted(f for f in os.listdir(HERE) if f.endswith(".npz")))


if __name__ == "__main__":
    main()
