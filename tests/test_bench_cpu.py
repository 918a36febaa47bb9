"""bench.py's host-side logic, with no GPU: the FLOP accounting of both
workloads, the clock record (throttle reasons and the loaded-sample filter
over nvidia-smi lines), the warm-up floor, and the reference arm's JSON line
(the CPU restatement of the reference's fp32 path on a row sample)."""
import json
import os
import subprocess
import sys

import pytest

import bench

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_flop_accounting_of_both_workloads():
    # 6 M (2 H D + H Dout): the reference's accounting (results_fused_forward.md:75)
    assert bench.flops_fwd_bwd(**bench.CFG) == pytest.approx(10.2991e12, rel=1e-4)
    assert bench.flops_fwd_bwd(**bench.CFG5) == pytest.approx(277.08e12, rel=1e-4)
    kf = bench.kernel_flops(**bench.CFG)
    six = ["gemm1_swiglu", "gemm2_y", "gradh_dswiglu_emit_h", "dw2_gemm", "dw1", "dx"]
    assert sum(kf[k] for k in six) == pytest.approx(bench.flops_fwd_bwd(**bench.CFG))
    for name, (cfg, metric, workload) in bench.WORKLOADS.items():
        assert workload.startswith(name)
        assert all(f"{k}={v}" in metric for k, v in cfg.items())


def _sample(sm, power, reasons=()):
    names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
    flags = ", ".join("Active" if n in reasons else "Not Active" for n in names)
    return f"0, {sm}, 1965, {power}, 0x0, {flags}"


def test_clock_summary_keeps_loaded_samples_and_their_reasons():
    clk = bench.ClockSampler(0)
    clk.lines = ([_sample(1965, 120.0)] * 3                                   # idle, before the region
                 + [_sample(1350, 980.0, ["sw_power_cap"])] * 5
                 + [_sample(1410, 960.0, ["sw_power_cap"])] * 4
                 + [_sample(1965, 150.0, ["hw_slowdown"])]                    # idle tail: not counted
                 + ["garbage line"])
    s = clk.summary()
    assert s["loaded_samples"] == 9 and s["samples"] == 13
    assert s["sm_mhz"] == 1350 and s["sm_max_mhz"] == 1965
    assert s["reasons"] == ["sw_power_cap"]


def test_clock_summary_without_samples_is_none():
    clk = bench.ClockSampler(0)
    clk.lines = []
    assert clk.summary() is None


def test_warmup_below_three_is_rejected():
    out = subprocess.run([sys.executable, os.path.join(REPO, "bench.py"), "--warmup", "2"],
                         capture_output=True, text=True, timeout=300)
    assert out.returncode != 0 and "--warmup must be >= 3" in out.stderr


def test_reference_arm_prints_one_contract_line():
    out = subprocess.run([sys.executable, os.path.join(REPO, "bench.py"), "--impl", "reference",
                          "--steps", "1", "--warmup", "3"], capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [ln for ln in out.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["metric"] == bench.METRIC and d["unit"] == "TFLOP/s"
    assert d["higher_is_better"] is True and d["value"] > 0
    assert {k: d["config"][k] for k in bench.CFG} == bench.CFG
    assert d["cpu_baseline"]["kind"] == "port" and d["cpu_baseline"]["value"] == d["value"]
    assert d["e2e"] == {"value": d["value"], "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}


def test_launch_labels_of_both_dw2_modes():
    fwd = ["swiglu_b200_fused_matmul_swiglu_save_preact", "swiglu_b200_matmul_tiled"]
    emit = fwd + ["swiglu_b200_bwd_grad_preact_inplace_emit_h"] + ["swiglu_b200_matmul_tiled"] * 3
    pro = fwd + ["swiglu_b200_bwd_dw2", "swiglu_b200_bwd_grad_preact_inplace"] + ["swiglu_b200_matmul_tiled"] * 2
    assert bench.label_launches(emit * 2) == ["gemm1_swiglu", "gemm2_y", "gradh_dswiglu_emit_h", "dw2_gemm",
                                              "dw1", "dx"] * 2
    assert bench.label_launches(pro * 2) == ["gemm1_swiglu", "gemm2_y", "dw2_hprologue", "gradh_dswiglu",
                                             "dw1", "dx"] * 2
    kf = bench.kernel_flops(**bench.CFG)
    for seq in (emit, pro):
        assert sum(kf[k] for k in bench.label_launches(seq)) == pytest.approx(bench.flops_fwd_bwd(**bench.CFG))


class _Ev:
    """A recorded event at time t (ms) on one stream."""

    def __init__(self, t):
        self.t = t

    def elapsed_time(self, other):
        return other.t - self.t


def test_tp_launch_sequence_times_and_idle_gaps():
    # Two steps of three launches: a (1 ms), b (2 ms) after 0.5 ms idle,
    # c (1 ms) after 0.25 ms idle; step 1's first launch after 0.75 ms idle.
    recs, t = [], 0.0
    for _ in range(2):
        for name, idle, run in (("a", 0.75, 1.0), ("b", 0.5, 2.0), ("c", 0.25, 1.0)):
            t += idle
            recs.append((name, _Ev(t), _Ev(t + run)))
            t += run
    seq = bench.tp_launch_sequence(recs, 2)
    assert [n for n, _, _ in seq] == ["a", "b", "c"]
    for (_, run, gap), (want_run, want_gap) in zip(seq, [(1.0, 0.75), (2.0, 0.5), (1.0, 0.25)]):
        assert run == pytest.approx(want_run) and gap == pytest.approx(want_gap)
    assert bench.tp_launch_sequence(recs[:5], 2) == []
