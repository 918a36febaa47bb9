"""SwiGLU-MLP fwd+bwd benchmark on B200 (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload: config 2 of the benchmark, one SwiGLU MLP block in bf16,
M=11136 D=3584 H=14336 Dout=3584, forward + recompute backward through the
public API (SwiGLUMLPCustom / SwiGLUMemoryOptimizedFunction), seeded synthetic
inputs (x, grad_y ~ N(0,1); W ~ N(0, fan_in^-1/2)). FLOPs per step
6*M*(2H*D + H*Dout) = 10.2991 TFLOP (recompute and pointwise work not counted).

  value      device-timed whole-job TFLOP/s, inputs resident in HBM (every
             step's working set, >= 1.5 GB, exceeds the 126 MB L2)
  kernels_ms each native kernel's mean device time inside those same timed
             steps (CUDA events around every launch on its stream)
  e2e        same metric through the public API with host buffers: pinned
             x and grad_y copied in and grad_x copied out every step
  roofline   the dominant kernel's algorithmic TFLOP/s vs measured bf16 peak
  same_box   the reference's recompute algorithm (cuBLAS GEMMs + Inductor
             pointwise) on the same GPU, burst and sustained, beside ours
  cpu_baseline  the reference's pure-PyTorch fp32 path (CPU restatement),
             timed on this host on a bounded row sample of the same shapes

For N > 1 the block is tensor-parallel (tp.py): W1 column-sharded with
left/gate pairs together, W2 row-sharded, x/grad_y all-gathered and the
partial y / grad_x reduce-scattered over NCCL; the total workload stays
config 2 (strong scaling).
"""
from __future__ import annotations

import argparse
import json
import os
import re
import statistics
import subprocess
import sys
import time

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(REPO, "swiglu-recompute_b200"))
sys.path.insert(0, REPO)

import torch  # noqa: E402

CFG = dict(M=11136, D=3584, H=14336, Dout=3584)
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
METRIC = "SwiGLU-MLP fwd+bwd TFLOP/s (bf16, M=11136 D=3584 H=14336 Dout=3584)"
# The tensor-parallel configuration (Llama-3-70B MLP shape, 1/2/4/8 GPUs):
# `--workload cfg5`, measured beside the bench line, not instead of it.
CFG5 = dict(M=65536, D=8192, H=28672, Dout=8192)
WORKLOADS = {
    "cfg2": (CFG, METRIC, "cfg2: one SwiGLU MLP block fwd+bwd"),
    "cfg5": (CFG5, "SwiGLU-MLP fwd+bwd TFLOP/s (bf16, M=65536 D=8192 H=28672 Dout=8192)",
             "cfg5: one SwiGLU MLP block fwd+bwd, Llama-3-70B MLP shape"),
}


def flops_fwd_bwd(M, D, H, Dout):
    return 6.0 * M * (2 * H * D + H * Dout)


def load_peaks():
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return d, "measured"
    return FALLBACK_PEAKS, "fallback"


def profile_traffic(kernel):
    """Per-launch DRAM bytes (read + write) of `kernel` from the committed ncu
    summary profiles/traffic.md, or None."""
    p = os.path.join(REPO, "profiles", "traffic.md")
    if not os.path.exists(p):
        return None
    with open(p) as f:
        m = re.search(r"traffic_bytes_per_launch\[" + re.escape(kernel) + r"\]:\s*([0-9.eE+]+)", f.read())
    return float(m.group(1)) if m else None


# ---------------------------------------------------------------- clocks
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "25", "-i", str(self.index)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        self.lines = []
        if self.proc is not None:
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [ln for ln in out.splitlines() if ln.strip()]

    def summary(self):
        """Median SM clock, power and the throttle reasons seen over the samples
        taken under load (power draw >= 60 % of the highest sample; the sampler
        also runs a little before and after the timed region)."""
        rows, mx = [], None
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in getattr(self, "lines", []):
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm, pw = float(parts[1]), float(parts[3])
                mx = float(parts[2])
            except ValueError:
                continue
            rows.append((sm, pw, {n for n, v in zip(names, parts[5:9]) if v.lower() == "active"}))
        if not rows:
            return None
        top = max(r[1] for r in rows)
        loaded = [r for r in rows if r[1] >= 0.6 * top]
        reasons = set().union(*(r[2] for r in loaded))
        return {"sm_mhz": statistics.median(r[0] for r in loaded), "sm_max_mhz": mx,
                "power_w": round(statistics.median(r[1] for r in loaded), 1), "reasons": sorted(reasons),
                "samples": len(rows), "loaded_samples": len(loaded)}


# ------------------------------------------------------------- CPU arm
def cpu_reference_sample(seconds=12.0, rows=256, cfg=CFG):
    """The reference's fp32 path (oracle restatement) on this host's cores, on a
    `rows`-row slice of `cfg`'s shapes. Returns (TFLOP/s, cores, sample)."""
    from oracle import swiglu_oracle as O

    D, H, Dout = cfg["D"], cfg["H"], cfg["Dout"]
    torch.set_num_threads(os.cpu_count() or 1)
    x, w1, w2, gy = O.make_inputs(rows, D, H, Dout, seed=0, dtype=torch.float32)
    O.mlp_forward_backward(x[:16], w1, w2, gy[:16])            # warm-up
    fl = flops_fwd_bwd(rows, D, H, Dout)
    times = []
    t_end = time.perf_counter() + seconds
    while time.perf_counter() < t_end or len(times) < 2:
        t0 = time.perf_counter()
        O.mlp_forward_backward(x, w1, w2, gy)
        times.append(time.perf_counter() - t0)
    best = min(times)
    return fl / best / 1e12, torch.get_num_threads(), (
        f"fp32 fwd+bwd of {rows} of {cfg['M']} rows at D={D} H={H} Dout={Dout}, "
        f"best of {len(times)} (wall clock)")


def run_reference_arm(args, rank, world):
    if rank != 0:
        return
    cfg, metric, workload = WORKLOADS[args.workload]
    tf, cores, sample = cpu_reference_sample(seconds=max(6.0, 2.0 * (args.steps + args.warmup)), cfg=cfg)
    line = {
        "impl": "reference", "metric": metric, "value": round(tf, 4), "unit": "TFLOP/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "higher_is_better": True, "dtype": "f32", "data": "synthetic",
        "config": {"workload": workload + ", reference fp32 path on the host cores (row sample)", **cfg,
                   "parallelism": "one host process"},
        "cpu_baseline": {"value": round(tf, 4), "unit": "TFLOP/s", "cores": cores, "kind": "port",
                         "sample": sample},
        "e2e": {"value": round(tf, 4), "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "vs_baseline": None,
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------- GPU arm
def _inputs(dev, dtype=torch.bfloat16, cfg=CFG):
    """Config 2: drawn on the host (the bits every backend and test sees).
    Config 5 (7 GiB of f32 draws): drawn on `dev`, same distributions."""
    from swiglu_b200.synthetic import make_inputs, make_inputs_on_device
    if cfg is CFG5:
        return make_inputs_on_device(cfg["M"], cfg["D"], cfg["H"], cfg["Dout"], dev, seed=0, dtype=dtype)
    return make_inputs(cfg["M"], cfg["D"], cfg["H"], cfg["Dout"], seed=0, dtype=dtype)


def label_launches(names):
    """Kernel names of the step's native launches, in launch order, from the
    entry points the launch trace records (swiglu_b200.ops.trace_launches).
    One step: GEMM1+SwiGLU, y; then either grad_h+dSwiGLU writing h and the
    dW2 GEMM on it ("emit_h"), or the dW2 kernel with the h prologue and
    grad_h+dSwiGLU ("prologue"); then dW1 and dx."""
    out, fwd, dw2_pending, bwd_mm = [], True, False, 0
    for n in names:
        if n == "swiglu_b200_fused_matmul_swiglu_save_preact":
            out.append("gemm1_swiglu")
            fwd, dw2_pending, bwd_mm = True, False, 0
        elif n == "swiglu_b200_bwd_dw2":
            out.append("dw2_hprologue")
            fwd = False
        elif n in ("swiglu_b200_bwd_grad_preact_inplace_emit_h", "swiglu_b200_bwd_grad_preact_inplace"):
            emit = n.endswith("emit_h")
            out.append("gradh_dswiglu_emit_h" if emit else "gradh_dswiglu")
            fwd, dw2_pending, bwd_mm = False, emit, 0
        elif n == "swiglu_b200_matmul_tiled":
            if fwd:
                out.append("gemm2_y")
            elif dw2_pending:
                out.append("dw2_gemm")
                dw2_pending = False
            else:
                out.append(("dw1", "dx")[min(bwd_mm, 1)])
                bwd_mm += 1
        else:
            out.append(n)
    return out


def traced_kernel_ms(records, steps):
    """{kernel: mean ms per step} of the launches recorded over `steps` steps."""
    labels = label_launches([r[0] for r in records])
    acc = {}
    for lab, (_, e0, e1) in zip(labels, records):
        acc[lab] = acc.get(lab, 0.0) + e0.elapsed_time(e1)
    return {k: v / steps for k, v in acc.items()}


def tp_launch_sequence(records, steps):
    """[(entry point, mean ms, mean idle ms before it)] of one step's native
    launches in launch order, from `steps` steps of launch records on one
    stream (every step makes the same launches; the first launch's idle time
    is taken from the previous step's last launch, so step 0 does not count
    it); [] if the records do not split evenly."""
    if not records or len(records) % steps:
        return []
    per = len(records) // steps
    out = []
    for i in range(per):
        name = records[i][0]
        run = sum(records[s * per + i][1].elapsed_time(records[s * per + i][2]) for s in range(steps)) / steps
        prev = [(s * per + i - 1) for s in range(steps) if s * per + i >= 1]
        gap = sum(records[j][2].elapsed_time(records[j + 1][1]) for j in prev) / max(1, len(prev))
        out.append((name, run, gap))
    return out


def kernel_flops(M, D, H, Dout):
    g1 = 2.0 * M * D * 2 * H
    g2 = 2.0 * M * H * Dout
    return {"gemm1_swiglu": g1, "gemm2_y": g2, "gradh_dswiglu_emit_h": g2, "gradh_dswiglu": g2,
            "dw2_gemm": g2, "dw2_hprologue": g2, "dw1": g1, "dx": g1}


def run_kernel_only(args):
    """Launch one kernel of the step `args.iters` times at config-2 shapes
    (the case the committed ncu summaries under profiles/ are taken on)."""
    from swiglu_b200 import ops
    from swiglu_b200.ops import LAYOUT_STD, W1_ROWS

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    M, D, H, Dout = CFG["M"], CFG["D"], CFG["H"], CFG["Dout"]
    x, w1, w2, gy = (t.to(dev) for t in _inputs(dev))
    preact, h = ops.swiglu_fwd(x, w1, w_form=W1_ROWS, layout=LAYOUT_STD, h_from_rounded=True)
    k = args.kernel
    gm = {} if args.group_m is None else {"group_size_m": args.group_m}
    calls = {
        "gemm1": lambda: ops.swiglu_fwd(x, w1, w_form=W1_ROWS, layout=LAYOUT_STD, h_from_rounded=True, **gm),
        "y": lambda: ops.matmul(h, w2, a_t=False, b_t=True, **gm),
        "dw2": lambda: ops.bwd_dw2(gy, preact, layout=LAYOUT_STD),
        "dw2gemm": lambda: ops.matmul(gy, h, a_t=True, b_t=False, **gm),
        # in place on a scratch copy so repeated launches see the same input
        "gradh": lambda: ops.bwd_grad_preact_inplace(gy, w2, pre2, layout=LAYOUT_STD, h_out=h),
        "dw1": lambda: ops.matmul(preact, x, a_t=True, b_t=False, tile_n=512, **gm),
        "dx": lambda: ops.matmul(preact, w1, a_t=False, b_t=False, tile_n=512, **gm),
    }
    pre2 = torch.empty_like(preact) if k == "gradh" else None
    fl = kernel_flops(M, D, H, Dout)[{"gemm1": "gemm1_swiglu", "y": "gemm2_y", "dw2": "dw2_hprologue",
                                      "dw2gemm": "dw2_gemm", "gradh": "gradh_dswiglu_emit_h", "dw1": "dw1",
                                      "dx": "dx"}[k]]
    times = []
    for _ in range(args.iters):
        if pre2 is not None:
            pre2.copy_(preact)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        calls[k]()
        e1.record()
        torch.cuda.synchronize()
        times.append(e0.elapsed_time(e1))
    assert ops.device_status(0) == 0
    best = min(times)
    print(json.dumps({"kernel": k, "ms": round(best, 4), "tflops": round(fl / best / 1e9, 1),
                      "times_ms": [round(t, 4) for t in times]}), flush=True)


REFERENCE_STACK_PEAK_MIB = {1: 2275, 2: 2961, 4: 4334, 8: 7078, 16: 12567}   # results_b200.md:38-42
REFERENCE_STACK_MS = {1: 8.0, 2: 16.3, 4: 32.9, 8: 55.7, 16: 104.7}             # results_b200.md:38-42


def _event_ms_interleaved(fns, reps=12, warm=3):
    """Minimum CUDA-event time of one call of each of `fns` ({name: fn}); the
    variants take turns call by call, so each sees the same power and
    thermal state (each call's operands exceed the 126 MB L2, so no flush)."""
    for fn in fns.values():
        for _ in range(warm):
            fn()
    torch.cuda.synchronize()
    best = {k: float("inf") for k in fns}
    for _ in range(reps):
        for k, fn in fns.items():
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            fn()
            e1.record()
            torch.cuda.synchronize()
            best[k] = min(best[k], e0.elapsed_time(e1))
    return best


def run_fwd_sweep(args):
    """Forward-only W1 projection + SwiGLU, the benchmark's forward-only configuration (packed weight,
    D=4096 H=14336, M in {1024, 4096, 16384, 65536}) and the config-2 shape:
    this library's fused kernel saving preact and h, its no-save form (h only),
    cuBLAS GEMM + compiled SwiGLU, cuBLAS GEMM alone (the comparison of
    results_fused_forward.md:75-80). One JSON line per shape; FLOPs 4*M*D*H."""
    import torch.nn.functional as F
    from swiglu_b200.synthetic import make_inputs
    from swiglu_b200 import ops
    from swiglu_b200.ops import LAYOUT_PACKED128, W1_T

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    for M, D, H in [(1024, 4096, 14336), (4096, 4096, 14336), (16384, 4096, 14336), (65536, 4096, 14336),
                    (11136, 3584, 14336)]:
        x, w1, _, _ = make_inputs(M, D, H, 8, seed=0, dtype=torch.bfloat16)
        x, w1 = x.to(dev), w1.to(dev)
        wt = w1.t().contiguous()                                     # [D, 2H] standard
        wp = ops.pack_chunked(wt, 128, unpack=False)                 # [D, 2H] packed
        act = torch.compile(lambda p, n=H: F.silu(p[:, n:]) * p[:, :n])
        fns = {
            "fused_save_packed": lambda: ops.swiglu_fwd(x, wp, w_form=W1_T, layout=LAYOUT_PACKED128,
                                                        h_from_rounded=False),
            "fused_nosave_packed": lambda: ops.swiglu_fwd(x, wp, w_form=W1_T, layout=LAYOUT_PACKED128,
                                                          h_from_rounded=False, want_preact=False),
            "cublas_gemm_plus_compiled_act": lambda: act(x @ wt),
            "cublas_gemm": lambda: x @ wt,
        }
        ms = _event_ms_interleaved(fns)
        fl = 4.0 * M * D * H
        print(json.dumps({"sweep": "fwd", "M": M, "D": D, "H": H, "ms": {k: round(v, 4) for k, v in ms.items()},
                          "tflops": {k: round(fl / (v * 1e-3) / 1e12, 1) for k, v in ms.items()}}), flush=True)
        del x, w1, wt, wp
        torch.cuda.empty_cache()
    from swiglu_b200.ops import device_status
    assert device_status(0) == 0


def run_stack_sweep(args):
    """Stacked depth, the benchmark's depth configuration: N in {1, 2, 4, 8, 16} config-2 blocks,
    peak memory and ms per fwd+bwd as the reference measures them, for the
    recompute module, the full-checkpoint module and, on the same GPU, the
    torch.compile'd standard MLP (cuBLAS GEMMs + Inductor pointwise, the
    reference's fair baseline) and the reference's recompute algorithm
    (reference_recompute_module). One JSON line per N."""
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    for n in (1, 2, 4, 8, 16):
        peak, ms = stacked_depth(n, dev)
        peak_fc, ms_fc = stacked_depth(n, dev, module="SwiGLUMLPFullCheckpoint")
        peak_gt, ms_gt = stacked_depth(n, dev, module="SwiGLUMLPGroundTruth", compile_model=True)
        peak_ra, ms_ra = stacked_depth(n, dev, module=reference_recompute_module)
        torch._dynamo.reset()
        _REF_HELPERS.clear()
        print(json.dumps({"sweep": "stack", "n_blocks": n,
                          "recompute": {"peak_mib": round(peak, 1), "ms_per_step": round(ms, 3)},
                          "full_checkpoint": {"peak_mib": round(peak_fc, 1), "ms_per_step": round(ms_fc, 3)},
                          "standard_mlp_compiled_same_box": {"peak_mib": round(peak_gt, 1),
                                                             "ms_per_step": round(ms_gt, 3)},
                          "reference_algorithm_same_box": {"peak_mib": round(peak_ra, 1),
                                                           "ms_per_step": round(ms_ra, 3)},
                          "reference_recompute": {"peak_mib": REFERENCE_STACK_PEAK_MIB[n],
                                                  "ms_per_step": REFERENCE_STACK_MS[n]}}), flush=True)


def run_energy_sweep(args, seconds=2.5):
    """Energy per launch of each native kernel of the config-2 step, alone and
    back to back for `seconds` (long enough for the 1 kW power cap to set the
    clock), on both pair-tile widths where the library chooses one, and of
    cuBLAS GEMMs of the same shapes: NVML's total-energy counter over the
    run, ms per launch by CUDA events. One JSON line per kernel; not the
    bench line."""
    import pynvml
    from swiglu_b200 import _lib, ops
    from swiglu_b200.ops import LAYOUT_STD, W1_ROWS

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    pynvml.nvmlInit()
    hd = pynvml.nvmlDeviceGetHandleByIndex(0)
    M, D, H, Dout = CFG["M"], CFG["D"], CFG["H"], CFG["Dout"]
    x, w1, w2, gy = (t.to(dev) for t in _inputs(dev))
    preact, h = ops.swiglu_fwd(x, w1, w_form=W1_ROWS, layout=LAYOUT_STD, h_from_rounded=True)
    pre2 = preact.clone()
    kf = kernel_flops(M, D, H, Dout)

    def path(fn, p):
        def run():
            _lib.set_gemm_path(p)
            try:
                return fn()
            finally:
                _lib.set_gemm_path(0)
        return run

    g1 = lambda: ops.swiglu_fwd(x, w1, w_form=W1_ROWS, layout=LAYOUT_STD, h_from_rounded=True)  # noqa: E731
    gh = lambda: ops.bwd_grad_preact_inplace(gy, w2, pre2, layout=LAYOUT_STD)  # noqa: E731
    cases = [
        ("gemm1_swiglu 256x256", g1, kf["gemm1_swiglu"]),
        ("gemm1_swiglu 256x512", path(g1, 3), kf["gemm1_swiglu"]),
        ("cublas x.W1^T", lambda: x @ w1.t(), kf["gemm1_swiglu"]),
        ("gemm2_y 256x256", lambda: ops.matmul(h, w2, a_t=False, b_t=True, tile_n=256), kf["gemm2_y"]),
        ("gemm2_y 256x512", lambda: ops.matmul(h, w2, a_t=False, b_t=True, tile_n=512), kf["gemm2_y"]),
        ("cublas h.W2^T", lambda: h @ w2.t(), kf["gemm2_y"]),
        ("gradh_dswiglu 256x256", gh, kf["gradh_dswiglu"]),
        ("gradh_dswiglu 256x512", path(gh, 3), kf["gradh_dswiglu"]),
        ("cublas grad_y.W2 (no epilogue)", lambda: gy @ w2, kf["gradh_dswiglu"]),
        ("dw2_hprologue", lambda: ops.bwd_dw2(gy, preact, layout=LAYOUT_STD), kf["dw2_hprologue"]),
        ("dw2_gemm 256x256", lambda: ops.matmul(gy, h, a_t=True, b_t=False, tile_n=256), kf["dw2_gemm"]),
        ("dw2_gemm 256x512", lambda: ops.matmul(gy, h, a_t=True, b_t=False, tile_n=512), kf["dw2_gemm"]),
        ("cublas grad_y^T.h", lambda: gy.t() @ h, kf["dw2_gemm"]),
        ("dw1 256x512", lambda: ops.matmul(preact, x, a_t=True, b_t=False, tile_n=512), kf["dw1"]),
        ("cublas preact^T.x", lambda: preact.t() @ x, kf["dw1"]),
        ("dx 256x512", lambda: ops.matmul(preact, w1, a_t=False, b_t=False, tile_n=512), kf["dx"]),
        ("cublas preact.W1", lambda: preact @ w1, kf["dx"]),
    ]
    for name, fn, fl in cases:
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        time.sleep(1.5)                                     # let the power average fall back
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        n, clocks = 0, []
        t0 = time.perf_counter()
        en0 = pynvml.nvmlDeviceGetTotalEnergyConsumption(hd)
        e0.record()
        while time.perf_counter() - t0 < seconds:
            for _ in range(20):
                fn()
            n += 20
            clocks.append(pynvml.nvmlDeviceGetClockInfo(hd, pynvml.NVML_CLOCK_SM))
            torch.cuda.synchronize()
        e1.record()
        torch.cuda.synchronize()
        en1 = pynvml.nvmlDeviceGetTotalEnergyConsumption(hd)
        ms = e0.elapsed_time(e1) / n
        joules = (en1 - en0) / 1000.0 / n
        clocks.sort()
        print(json.dumps({"sweep": "energy", "kernel": name, "launches": n, "ms": round(ms, 4),
                          "tflops": round(fl / ms / 1e9, 1), "mJ_per_launch": round(joules * 1e3, 1),
                          "pJ_per_flop": round(joules / fl * 1e12, 4), "watts": round(joules / (ms * 1e-3), 1),
                          "sm_mhz_median": clocks[len(clocks) // 2]}), flush=True)
    assert ops.device_status(0) == 0


def run_power_sweep(args):
    """Sustained load (about 3 s per arm, long enough for the 1 kW power cap to
    set the clock) on one GPU at `--workload`'s shape: the six-kernel step with
    the tile widths the library picks, with every GEMM on 256 x 256 and on
    256 x 512 tiles, and the eager PyTorch MLP (cuBLAS GEMMs + pointwise) for
    comparison. Per arm: ms per step and per kernel over the last two thirds
    of the steps (CUDA events) and the sampled clocks. One JSON line per arm;
    not the bench line."""
    from swiglu_b200 import _lib, ops
    from swiglu_b200.ops import LAYOUT_STD, W1_ROWS

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    cfg, _, workload = WORKLOADS[args.workload]
    M, D, H, Dout = cfg["M"], cfg["D"], cfg["H"], cfg["Dout"]
    x, w1, w2, gy = (t.to(dev) for t in _inputs(dev, cfg=cfg))
    fl = flops_fwd_bwd(M, D, H, Dout)
    names = ["gemm1_swiglu", "gemm2_y", "gradh_dswiglu_emit_h", "dw2_gemm", "dw1", "dx"]

    def ours(ev):
        ev[0].record()
        preact, h = ops.swiglu_fwd(x, w1, w_form=W1_ROWS, layout=LAYOUT_STD, h_from_rounded=True)
        ev[1].record()
        y = ops.matmul(h, w2, a_t=False, b_t=True)
        ev[2].record()
        del y
        ops.bwd_grad_preact_inplace(gy, w2, preact, layout=LAYOUT_STD, h_out=h)
        ev[3].record()
        dw2 = ops.matmul(gy, h, a_t=True, b_t=False)
        ev[4].record()
        del h
        dw1 = ops.matmul(preact, x, a_t=True, b_t=False, tile_n=512)
        ev[5].record()
        dx = ops.matmul(preact, w1, a_t=False, b_t=False, tile_n=512)
        ev[6].record()
        return dw2, dw1, dx

    W1 = w1.detach().clone().requires_grad_(True)
    W2 = w2.detach().clone().requires_grad_(True)

    def torch_mlp(ev):
        ev[0].record()
        xi = x.detach().requires_grad_(True)
        left, gate = (xi @ W1.t()).chunk(2, dim=-1)
        y = (left * torch.nn.functional.silu(gate)) @ W2.t()
        out = torch.autograd.grad(y, [xi, W1, W2], gy)
        ev[6].record()
        return out

    est_ms = fl / 1.2e12   # one step at ~1.2 PFLOP/s
    arms = [("library", ours, 0), ("all_256x256", ours, 2), ("all_256x512", ours, 3),
            ("torch_eager_cublas", torch_mlp, 0)]
    for name, fn, path in arms:
        _lib.set_gemm_path(path)
        try:
            dummy = [torch.cuda.Event() for _ in range(7)]
            for _ in range(3):
                fn(dummy)
            torch.cuda.synchronize()
            n = max(9, int(3000.0 / est_ms))
            evs = [[torch.cuda.Event(enable_timing=True) for _ in range(7)] for _ in range(n)]
            with ClockSampler(0) as clk:
                time.sleep(0.3)
                for i in range(n):
                    fn(evs[i])
                torch.cuda.synchronize()
        finally:
            _lib.set_gemm_path(0)
        tail = evs[n // 3:]
        ms = sum(e[0].elapsed_time(e[6]) for e in tail) / len(tail)
        line = {"sweep": "power", "workload": workload, **cfg, "arm": name, "steps": n,
                "ms_per_step": round(ms, 4), "tflops": round(fl / ms / 1e9, 1), "clocks": clk.summary()}
        if fn is ours:
            line["kernels_ms"] = {k: round(sum(e[i].elapsed_time(e[i + 1]) for e in tail) / len(tail), 4)
                                  for i, k in enumerate(names)}
        print(json.dumps(line), flush=True)
    assert ops.device_status(0) == 0


def stacked_depth(n_blocks, dev, reps=3, iters=3, module="SwiGLUMLPCustom", compile_model=False):
    """Peak allocated-memory delta (MiB) and ms per fwd+bwd of `n_blocks`
    stacked config-2 blocks, measured as the reference's stacked-depth
    benchmark does (bench_stacked_blocks.py:55-102): two warm-up steps, then
    per rep reset the peak counter, record the base allocation, run forward
    through all blocks plus one autograd.grad, take peak - base; min over reps.
    Block i's weights are seeded with seed 1 + i. `module` names a module
    class of swiglu_recompute, or is a callable (D, H, Dout, w1, w2, dev) ->
    block such as reference_recompute_module. `compile_model` wraps the
    stack in torch.compile (the reference's fair baseline does so for the
    standard MLP, bench_fair_compile.py:45)."""
    import swiglu_recompute as SR
    from swiglu_b200.synthetic import make_inputs

    M, D, H = CFG["M"], CFG["D"], CFG["H"]
    blocks = []
    for i in range(n_blocks):
        _, w1, w2, _ = make_inputs(1, D, H, D, seed=1 + i, dtype=torch.bfloat16)
        if callable(module):
            blocks.append(module(D, H, D, w1, w2, dev))
            continue
        b = getattr(SR, module)(D, H, D, dtype=torch.bfloat16).to(dev)
        with torch.no_grad():
            b.w1.copy_(w1)
            b.w2.copy_(w2)
        blocks.append(b)
    model = torch.nn.Sequential(*blocks)
    params = list(model.parameters())
    if compile_model:
        model = torch.compile(model)
    x0, _, _, _ = make_inputs(M, D, 1, 1, seed=0, dtype=torch.bfloat16)
    g = torch.Generator().manual_seed(7)
    x0 = x0.to(dev)
    gout = torch.randn(M, D, generator=g).to(torch.bfloat16).to(dev)

    def step():
        x = x0.detach().requires_grad_(True)
        y = model(x)
        return torch.autograd.grad(y, [x] + params, gout)

    for _ in range(2):
        step()
    torch.cuda.synchronize()
    best = None
    for _ in range(reps):
        torch.cuda.synchronize()
        torch.cuda.empty_cache()
        torch.cuda.reset_peak_memory_stats(dev)
        base = torch.cuda.memory_allocated(dev)
        grads = step()
        torch.cuda.synchronize()
        peak = torch.cuda.max_memory_allocated(dev) - base
        del grads
        best = peak if best is None else min(best, peak)
    times = []
    for _ in range(reps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(iters):
            step()
        e1.record()
        torch.cuda.synchronize()
        times.append(e0.elapsed_time(e1) / iters)
    del model, blocks, params
    torch.cuda.empty_cache()
    return best / 2 ** 20, min(times)


def e2e_pipelined(model, params, x, gy, dev, args):
    """Time `args.steps` steps through the public module API with host I/O.
    Returns (ms per step, H2D bytes per step, D2H bytes per step)."""
    M, D = x.shape
    x_h = [x.clone().pin_memory() for _ in range(2)]
    gy_h = [gy.clone().pin_memory() for _ in range(2)]
    dx_h = [torch.empty((M, D), dtype=torch.bfloat16).pin_memory() for _ in range(2)]
    x_d = [torch.empty_like(x, device=dev) for _ in range(2)]
    gy_d = [torch.empty_like(gy, device=dev) for _ in range(2)]
    comp = torch.cuda.current_stream(dev)
    copy = torch.cuda.Stream(dev)
    loaded = [torch.cuda.Event() for _ in range(2)]
    consumed = [torch.cuda.Event() for _ in range(2)]
    done = [torch.cuda.Event() for _ in range(2)]

    def load(i):
        s = i % 2
        with torch.cuda.stream(copy):
            copy.wait_event(consumed[s])
            x_d[s].copy_(x_h[s], non_blocking=True)
            gy_d[s].copy_(gy_h[s], non_blocking=True)
            loaded[s].record(copy)

    def run(nsteps):
        for s in range(2):
            consumed[s].record(comp)
        load(0)
        for i in range(nsteps):
            s = i % 2
            if i + 1 < nsteps:
                load(i + 1)
            comp.wait_event(loaded[s])
            xi = x_d[s].requires_grad_(True)
            gx = torch.autograd.grad(model(xi), [xi] + params, gy_d[s])[0]
            x_d[s].requires_grad_(False)
            done[s].record(comp)
            with torch.cuda.stream(copy):
                copy.wait_event(done[s])
                dx_h[s].copy_(gx, non_blocking=True)
                gx.record_stream(copy)
            consumed[s].record(comp)

    run(max(2, args.warmup // 2))
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(comp)
    run(args.steps)
    comp.wait_stream(copy)
    e1.record(comp)
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / args.steps, x.numel() * 2 + gy.numel() * 2, M * D * 2


_REF_HELPERS = []


def _reference_helpers():
    """The reference's two pointwise helpers (swiglu_recompute.py:26-49),
    compiled by Inductor once per process."""
    if not _REF_HELPERS:
        import torch.nn.functional as F

        @torch.compile
        def fwd_logic(preact):
            left, gate = preact.chunk(2, dim=-1)
            return left * F.silu(gate)

        @torch.compile
        def bwd_logic(preact, grad_h):
            left, gate = preact.chunk(2, dim=-1)
            sig = torch.sigmoid(gate)
            silu = gate * sig
            dsilu = sig + silu * (1.0 - sig)
            return torch.cat([grad_h * silu, grad_h * left * dsilu], dim=-1)

        _REF_HELPERS.extend([fwd_logic, bwd_logic])
    return _REF_HELPERS[0], _REF_HELPERS[1]


def reference_recompute_module(D, H, Dout, w1, w2, dev):
    """The reference's recompute MLP (swiglu_recompute.py:26-98) restated in
    torch ops, for a same-GPU comparison arm: cuBLAS GEMMs in the
    Function's order, and its two pointwise helpers compiled by Inductor as
    the reference compiles them (@torch.compile, :26 and :33). Not the
    reference's own file (it is not on the GPU box); the reference's Triton
    fused forwards need their source and are not run. Every block built here
    shares one pair of compiled helpers, as the reference's module-level
    functions are shared."""
    fwd_logic, bwd_logic = _reference_helpers()

    class Fn(torch.autograd.Function):
        @staticmethod
        def forward(ctx, x, W1, W2):
            preact = x @ W1.t()
            ctx.save_for_backward(x, W1, W2, preact)
            return fwd_logic(preact) @ W2.t()

        @staticmethod
        def backward(ctx, gy):
            x, W1, W2, preact = ctx.saved_tensors
            h = fwd_logic(preact)
            gw2 = gy.t() @ h
            gp = bwd_logic(preact, gy @ W2)
            return gp @ W1, gp.t() @ x, gw2

    class Module(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.w1 = torch.nn.Parameter(w1.to(dev, torch.bfloat16).clone())
            self.w2 = torch.nn.Parameter(w2.to(dev, torch.bfloat16).clone())

        def forward(self, x):
            return Fn.apply(x, self.w1, self.w2)

    return Module()


def _timed_steps(step, steps, st):
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record(st)
    for _ in range(steps):
        step()
    e1.record(st)
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / steps


def _sustained_ms(step, steps, st, seconds, est_ms):
    """ms per step over `steps` steps after `seconds` of back-to-back steps
    (long enough for the 1 kW power cap to settle the clock)."""
    for _ in range(max(1, int(seconds * 1e3 / est_ms))):
        step()
    return _timed_steps(step, steps, st)


def run_ours_single(args):
    import swiglu_recompute as SR
    from swiglu_b200 import ops

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    cfg, metric, workload = WORKLOADS[args.workload]
    M, D, H, Dout = cfg["M"], cfg["D"], cfg["H"], cfg["Dout"]
    x, w1, w2, gy = _inputs(dev, cfg=cfg)
    model = SR.SwiGLUMLPCustom(D, H, Dout, dtype=torch.bfloat16).to(dev)
    with torch.no_grad():
        model.w1.copy_(w1)
        model.w2.copy_(w2)
    params = list(model.parameters())
    xd, gyd = x.to(dev), gy.to(dev)

    def make_step(mod, prm):
        def step():
            xi = xd.detach().requires_grad_(True)
            y = mod(xi)
            return torch.autograd.grad(y, [xi] + prm, gyd)
        return step

    step = make_step(model, params)
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    assert ops.device_status(0) == 0, "kernel pipeline timeout during warm-up"

    # The timed steps, with every native launch bracketed by CUDA events on
    # its stream (ops.trace_launches): the per-kernel times below come from
    # these very steps, at these steps' clocks.
    st = torch.cuda.current_stream()
    records = []
    with ClockSampler(0) as clk:
        time.sleep(0.3)
        ops.trace_launches(records)
        try:
            ms = _timed_steps(step, args.steps, st)
        finally:
            ops.trace_launches(None)
    fl = flops_fwd_bwd(M, D, H, Dout)
    value = fl / (ms * 1e-3) / 1e12
    kt = traced_kernel_ms(records, args.steps)
    kf = kernel_flops(M, D, H, Dout)
    dom = max(kt, key=kt.get)
    launches = len(records)
    del records

    # The same step with dW2 in the other mode, timed the same way.
    other = "emit_h" if ops.dw2_mode() == "prologue" else "prologue"
    mode = ops.dw2_mode()
    ops.set_dw2_mode(other)
    try:
        for _ in range(2):
            step()
        ms_other = _timed_steps(step, args.steps, st)
    finally:
        ops.set_dw2_mode(mode)

    # The same step with the forward GEMMs on e4m3 operands (SwiGLUMLPFP8Forward:
    # per-row scaled x, W1, h, W2; bf16 recompute backward), and the inference
    # forward (no gradient: no preact saved) of both.
    fp8 = SR.SwiGLUMLPFP8Forward(D, H, Dout, dtype=torch.bfloat16).to(dev)
    with torch.no_grad():
        fp8.w1.copy_(model.w1)
        fp8.w2.copy_(model.w2)
    step8 = make_step(fp8, list(fp8.parameters()))
    for _ in range(2):
        step8()
    ms_fp8 = _timed_steps(step8, args.steps, st)
    with torch.no_grad():
        fwd_ms = {name: _timed_steps(lambda m=m: m(xd), args.steps, st) for name, m in (("bf16", model), ("e4m3", fp8))}
    del fp8, step8

    # End to end through the public API with host buffers: every step copies
    # its x and grad_y in from pinned host memory and its grad_x out, on a copy
    # stream that runs one step ahead (inputs of step i+1 and the output of
    # step i move while step i+1 / i computes), as a data loader would.
    e2e_ms, h2d, d2h = e2e_pipelined(model, params, x.cpu(), gy.cpu(), dev, args)

    peaks, peak_src = load_peaks()
    burst, sustained = float(peaks["bf16_tflops"]), float(peaks.get("bf16_tflops_sustained", peaks["bf16_tflops"]))
    ach = kf[dom] / (kt[dom] * 1e-3) / 1e12
    assert ops.device_status(0) == 0, "kernel pipeline timeout"

    line = {
        "metric": metric, "value": round(value, 2), "unit": "TFLOP/s", "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic" if cfg is CFG else "synthetic, drawn on the device",
        "config": {"workload": workload + ", recompute Function", **cfg, "parallelism": "tp1",
                   "dw2_mode": mode,
                   "l2": f"working set > L2 (preact alone {M * 2 * H * 2 / 2**20:.0f} MiB)"},
        "e2e": {"value": round(fl / (e2e_ms * 1e-3) / 1e12, 2), "unit": "TFLOP/s",
                "ms_per_step": round(e2e_ms, 4), "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
        "gpu_launches": launches,
        "frac_of_peak": {"burst": round(value / burst, 4), "sustained": round(value / sustained, 4),
                         "source": peak_src},
        # The timed steps are a short burst (clocks in "clocks"), so the
        # dominant kernel is held against the burst peak.
        "roofline": {"kernel": dom, "bound": "tensor", "achieved": round(ach, 2), "peak": burst,
                     "unit": "TFLOP/s", "frac": round(ach / burst, 4),
                     "frac_of_sustained_peak": round(ach / sustained, 4),
                     "traffic": profile_traffic(dom) if cfg is CFG else None,
                     "peak_kind": f"bf16_tflops, burst ({peak_src})"},
        "kernels_ms": {k: round(v, 4) for k, v in kt.items()},
        "kernels_sum_ms": round(sum(kt.values()), 4),
        "variants": {f"dw2_{other}": {"ms_per_step": round(ms_other, 4),
                                      "value": round(fl / (ms_other * 1e-3) / 1e12, 2)},
                     "fp8_forward": {"ms_per_step": round(ms_fp8, 4),
                                     "value": round(fl / (ms_fp8 * 1e-3) / 1e12, 2),
                                     "inference_forward_ms": {k: round(v, 4) for k, v in fwd_ms.items()},
                                     "note": "forward GEMMs on e4m3 operands with per-row scales, bf16 "
                                             "recompute backward; value counts the same FLOPs as the bf16 step"}},
        "clocks": clk.summary(),
    }
    if not args.no_same_box and cfg is CFG:
        line["same_box"] = same_box_comparison(args, make_step, model, params, w1, w2, dev, st, fl, ms)
    if not args.no_stack and cfg is CFG:
        peak, sms = stacked_depth(8, dev)
        line["stacked"] = {"n_blocks": 8, "peak_mib": round(peak, 1), "ms_per_step": round(sms, 3),
                           "dw2_mode": mode,
                           "reference_recompute_peak_mib": REFERENCE_STACK_PEAK_MIB[8],
                           "reference_recompute_ms_per_step": REFERENCE_STACK_MS[8],
                           "method": "max_memory_allocated - base over fwd+grad, min of 3 (as the reference)",
                           "not_counted": f"the stream-K workspace ({ops.STREAM_WORKSPACE_BYTES >> 20} MiB per "
                                          "stream, allocated on the stream's first use and held for the "
                                          "process) exists before base is taken"}
        ops.set_dw2_mode(other)
        try:
            peak_o, ms_o = stacked_depth(8, dev)
        finally:
            ops.set_dw2_mode(mode)
        line["variants"][f"dw2_{other}"]["stacked"] = {"n_blocks": 8, "peak_mib": round(peak_o, 1),
                                                       "ms_per_step": round(ms_o, 3)}
        peak_fc, ms_fc = stacked_depth(8, dev, module="SwiGLUMLPFullCheckpoint")
        line["stacked_full_checkpoint"] = {"n_blocks": 8, "peak_mib": round(peak_fc, 1),
                                           "ms_per_step": round(ms_fc, 3)}
        try:
            peak_r, ms_r = stacked_depth(8, dev, module=reference_recompute_module)
            line["stacked"]["reference_algorithm_same_box"] = {
                "peak_mib": round(peak_r, 1), "ms_per_step": round(ms_r, 3),
                "what": "8 blocks of reference_recompute_module (cuBLAS + Inductor), same method and GPU"}
        except Exception as e:  # the comparison arm must not take the bench line down
            line["stacked"]["reference_algorithm_same_box"] = {"error": f"{type(e).__name__}: {e}"[:300]}
    if not args.no_cpu_baseline and cfg is CFG:
        tf, cores, sample = cpu_reference_sample(seconds=args.cpu_seconds)
        line["cpu_baseline"] = {"value": round(tf, 4), "unit": "TFLOP/s", "cores": cores, "kind": "port",
                                "sample": sample}
    return line


def same_box_comparison(args, make_step, model, params, w1, w2, dev, st, fl, ms_burst):
    """The reference's recompute algorithm on this GPU (cuBLAS GEMMs + Inductor
    pointwise, reference_recompute_module) against this library's step:
    ms per step as a burst of `args.steps` steps and sustained (after
    `args.sustained_seconds` of back-to-back steps, at the power-capped
    clock), each with its sampled clocks."""
    out = {"reference_algorithm": "swiglu_recompute.py:58-78 in torch ops: cuBLAS bf16 GEMMs, "
                                  "Inductor-compiled pointwise helpers (torch.compile), same inputs",
           "triton_fused_forwards": "not run: the reference's Triton source does not travel to the GPU box"}
    try:
        ref = reference_recompute_module(model.dim, model.hidden_dim, model.out_dim, w1, w2, dev)
        ref_step = make_step(ref, list(ref.parameters()))
        for _ in range(max(3, args.warmup)):
            ref_step()                         # includes Inductor's compile on the first call
        torch.cuda.synchronize()
        time.sleep(1.0)
        with ClockSampler(0) as c0:
            time.sleep(0.3)
            ref_burst = _timed_steps(ref_step, args.steps, st)
        with ClockSampler(0) as c1:
            ref_sus = _sustained_ms(ref_step, args.steps, st, args.sustained_seconds, ref_burst)
        ours = make_step(model, params)
        with ClockSampler(0) as c2:
            ours_sus = _sustained_ms(ours, args.steps, st, args.sustained_seconds, ms_burst)
        del ref, ref_step
        torch.cuda.empty_cache()
    except Exception as e:  # the comparison arm must not take the bench line down
        out["error"] = f"{type(e).__name__}: {e}"[:300]
        return out
    out.update({
        "reference_burst_ms": round(ref_burst, 4), "reference_burst_clocks": c0.summary(),
        "reference_sustained_ms": round(ref_sus, 4), "reference_sustained_clocks": c1.summary(),
        "ours_burst_ms": round(ms_burst, 4),
        "ours_sustained_ms": round(ours_sus, 4), "ours_sustained_clocks": c2.summary(),
        "speedup_burst": round(ref_burst / ms_burst, 4), "speedup_sustained": round(ref_sus / ours_sus, 4),
        "sustained_seconds": args.sustained_seconds,
    })
    return out


def run_ours_tp(args):
    """Strong-scaling tensor-parallel run of one block of the workload's shape
    on WORLD_SIZE GPUs (one process per GPU, swiglu_b200.tp). Returns the JSON
    dict on rank 0, None elsewhere."""
    from datetime import timedelta

    import torch.distributed as dist
    from swiglu_b200 import ops
    from swiglu_b200.tp import FusedReduceScatter, SwiGLUMLPTensorParallel, tp_dw2_form

    cfg, metric, workload = WORKLOADS[args.workload]
    data = "synthetic" if cfg is CFG else "synthetic, drawn on the device"

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    assert world == args.gpus, f"--gpus {args.gpus} but WORLD_SIZE={world}"
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=180))
    try:
        M, D, H, Dout = cfg["M"], cfg["D"], cfg["H"], cfg["Dout"]
        assert M % world == 0 and H % world == 0
        x, w1, w2, gy = _inputs(dev, cfg=cfg)
        ms_rows = M // world
        # SWIGLU_TP_FUSED_RS: "1" each reduce-scatter rides on its GEMM where
        # the size rule (FusedReduceScatter.wants) says so, "0" NCCL only,
        # "y" / "all" the y / both reduce-scatters fused at any size.
        fuse_env = os.environ.get("SWIGLU_TP_FUSED_RS", "1")
        fused = fuse_env != "0"
        chunks = int(os.environ.get("SWIGLU_TP_CHUNKS", "1"))
        sm_reserve = int(os.environ.get("SWIGLU_SM_RESERVE", "0"))
        if sm_reserve:
            from swiglu_b200 import _lib
            _lib.set_sm_reserve(sm_reserve)
        frs = None
        if fused:
            frs = FusedReduceScatter()
            frs.always = {"y": ("y",), "all": ("y", "dx")}.get(fuse_env, ())
        model = SwiGLUMLPTensorParallel(D, H, Dout, dtype=torch.bfloat16, fused_rs=frs if fused else False,
                                        chunks=chunks).to(dev).load_full(w1, w2)
        params = list(model.parameters())
        x_l = x[rank * ms_rows:(rank + 1) * ms_rows].to(dev)
        gy_l = gy[rank * ms_rows:(rank + 1) * ms_rows].to(dev)
        del x, w1, w2, gy

        def step():
            xi = x_l.detach().requires_grad_(True)
            y = model(xi)
            return torch.autograd.grad(y, [xi] + params, gy_l)

        for _ in range(args.warmup):
            step()
        torch.cuda.synchronize()
        st = torch.cuda.current_stream()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        records = []
        with ClockSampler(local) as clk:
            time.sleep(0.3)
            dist.barrier()
            torch.cuda.synchronize()
            ops.trace_launches(records)
            try:
                e0.record(st)
                for _ in range(args.steps):
                    step()
                e1.record(st)
                torch.cuda.synchronize()
            finally:
                ops.trace_launches(None)
            dist.barrier()
        ms = torch.tensor([e0.elapsed_time(e1) / args.steps], device=dev)
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
        ms = ms.item()
        seq = tp_launch_sequence(records, args.steps)
        del records

        # End to end with host buffers: this rank's token shard in from pinned
        # host memory and its grad_x out, on a copy stream one step ahead of
        # the compute (the single-GPU bench's pipelined loop), max over ranks.
        x_host, gy_host = x_l.cpu(), gy_l.cpu()
        torch.cuda.synchronize()
        dist.barrier()
        e2e_ms, h2d, d2h = e2e_pipelined(model, params, x_host, gy_host, dev, args)
        e2e_ms = torch.tensor([e2e_ms], device=dev)
        dist.all_reduce(e2e_ms, op=dist.ReduceOp.MAX)
        e2e_ms = e2e_ms.item()
        status = torch.tensor([ops.device_status(local)], device=dev, dtype=torch.int64)
        dist.all_reduce(status, op=dist.ReduceOp.MAX)
        dist.barrier()
        # This library's launches per rank and step (GEMM1, y, grad_h, dW2,
        # dW1, dx per row piece, plus a signal and an owner-reduce kernel for
        # each GEMM that carries its reduce-scatter), as traced.
        launches = len(seq)
        how = {w: ("fused into the GEMM epilogue (f32 partials pushed over NVLink, summed by the owner)"
                   if frs is not None and frs.wants(k, w) else "NCCL reduce-scatter of f32 partials")
               for w, k in (("y", H // world), ("dx", 2 * H // world))}
        if rank != 0:
            return None
        fl = flops_fwd_bwd(M, D, H, Dout)
        peaks, src = load_peaks()
        peak = float(peaks.get("bf16_tflops_sustained", peaks["bf16_tflops"]))
        burst = float(peaks["bf16_tflops"])
        value = fl / (ms * 1e-3) / 1e12
        # GEMM1 (2.M.D.2H/t FLOPs per rank, over its row pieces) against the
        # burst peak, as in the 1-GPU line.
        g1_ms = sum(t for n, t, _ in seq if n == "swiglu_b200_fused_matmul_swiglu_save_preact")
        g1_ach = 2.0 * M * D * 2 * H / world / (g1_ms * 1e-3) / 1e12 if g1_ms else None
        kernels_sum = sum(t for _, t, _ in seq)
        return {
            "metric": metric, "value": round(value, 2), "unit": "TFLOP/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": data,
            "config": {"workload": workload + ", tensor parallel", **cfg,
                       "parallelism": f"tp{world}",
                       "reduce": how,
                       "chunks": chunks, "sm_reserve": sm_reserve,
                       "dw2_mode": tp_dw2_form(H // world, Dout,
                                               torch.cuda.get_device_properties(dev).multi_processor_count // 2),
                       "l2": "working set > L2"},
            "e2e": {"value": round(fl / (e2e_ms * 1e-3) / 1e12, 2), "unit": "TFLOP/s",
                    "ms_per_step": round(e2e_ms, 4),
                    "h2d_bytes_per_step": h2d * world, "d2h_bytes_per_step": d2h * world},
            "gpu_launches": launches * args.steps * world,
            "frac_of_peak": {"sustained": round(value / (peak * world), 4), "source": src},
            "roofline": ({"kernel": "gemm1_swiglu (per rank)", "bound": "tensor", "achieved": round(g1_ach, 2),
                          "peak": burst, "unit": "TFLOP/s", "frac": round(g1_ach / burst, 4), "traffic": None,
                          "peak_kind": f"bf16_tflops, burst ({src})"} if g1_ach else None),
            # Rank 0's native launches of one step in launch order: mean ms of
            # each and the compute stream's idle time before it (waiting on a
            # collective, or launch overhead), CUDA events on the compute
            # stream; the step time not covered by the launches is collective
            # time no kernel overlapped.
            "launch_sequence_ms": [[n, round(t, 4), round(g, 4)] for n, t, g in seq],
            "kernels_sum_ms": round(kernels_sum, 4),
            "device_status": int(status.item()),
            "clocks": clk.summary(),
        }
    finally:
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-stack", action="store_true", help="skip the 8-block stacked-depth memory run")
    ap.add_argument("--no-same-box", action="store_true",
                    help="skip the same-GPU comparison with the reference's recompute algorithm")
    ap.add_argument("--sustained-seconds", type=float, default=3.0,
                    help="back-to-back run before the sustained timings of the same-GPU comparison")
    ap.add_argument("--kernel", choices=["gemm1", "y", "dw2", "dw2gemm", "gradh", "dw1", "dx"],
                    help="launch only this kernel (profiling case)")
    ap.add_argument("--iters", type=int, default=5)
    ap.add_argument("--group-m", type=int, default=None,
                    help="with --kernel: L2 tile grouping in 128-row tiles (the reference's GROUP_SIZE_M)")
    ap.add_argument("--fwd-sweep", action="store_true",
                    help="forward-only W1 projection + SwiGLU vs cuBLAS, config 3 M sweep (not the bench line)")
    ap.add_argument("--stack-sweep", action="store_true",
                    help="stacked-depth memory and time at N = 1..16 blocks, config 4 (not the bench line)")
    ap.add_argument("--power-sweep", action="store_true",
                    help="sustained-load tile-width and PyTorch comparison at --workload (not the bench line)")
    ap.add_argument("--energy-sweep", action="store_true",
                    help="energy per launch of each kernel of the config-2 step under the power cap (not the bench line)")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="cfg2",
                    help="cfg2: the bench line's single block; cfg5: the tensor-parallel configuration "
                         "(M=65536 D=8192 H=28672 Dout=8192) at 1/2/4/8 GPUs")
    ap.add_argument("--gemm-path", type=int, choices=[0, 1, 2, 3], default=0,
                    help="tcgen05 kernel family: 0 by size, 1 single-SM, 2 CTA pair 256x256, 3 CTA pair 256x512")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))

    if args.gemm_path:
        from swiglu_b200 import _lib
        _lib.set_gemm_path(args.gemm_path)
    if os.environ.get("SWIGLU_DW2_MODE"):
        from swiglu_b200 import ops
        ops.set_dw2_mode(os.environ["SWIGLU_DW2_MODE"])
    if args.kernel:
        run_kernel_only(args)
        return
    if args.fwd_sweep:
        run_fwd_sweep(args)
        return
    if args.stack_sweep:
        run_stack_sweep(args)
        return
    if args.power_sweep:
        run_power_sweep(args)
        return
    if args.energy_sweep:
        run_energy_sweep(args)
        return
    if args.impl == "reference":
        run_reference_arm(args, rank, world)
        return
    if args.gpus == 1 and world == 1:
        line = run_ours_single(args)
        print(json.dumps(line), flush=True)
        return
    line = run_ours_tp(args)
    if line is not None:
        print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
