#!/usr/bin/env python
"""Benchmark of the quantized-linear hot path on B200.

Workload: one synthetic greedy decode step at batch 1 -- 48 layers of the
seven 4-bit g64 projections (q|k|v fused, o, gate|up fused, down) plus the quantized tied LM
head 262144 x 3840 with fused softcap + argmax; tensor-parallel over --gpus N (one process per
GPU, torchrun for N > 1). Seeded synthetic weights and activations (no checkpoint). Every rank
runs the step as ONE persistent-kernel launch (decode plan); for N > 1 the o/down partial sums
cross NVLink inside that kernel (peer stores) and the LM-head keys are combined there too.

value   = whole-job HBM GB/s of the quantized matmuls: 6,617,825,280 weight bytes streamed per
          token / device time of one decode step (CUDA graph replay, inputs already in HBM,
          weights 6.6 GB >> the 126 MB L2, so no flush is needed), max over ranks.
e2e     = the same metric through the public API with a host hidden state copied in (pinned H2D)
          and the token read back (D2H) inside the timed region, every step.
roofline: the dominant (only) kernel is the persistent decode kernel, one launch per step;
          achieved = the rank's algorithmic bytes per launch (its weight shards + activations) /
          the launch's CUDA-event duration (max over ranks); peak = MEASURED_PEAKS.json hbm_gbs.
qmatmul: BASELINE configs 1 and 2 on the standalone matmul entry point at N = 1: the up_proj
          15360 x 3840 at M = 1 and one layer's seven projections at M in {1, 2, 4, 8}, GB/s of
          algorithmic bytes, launches back to back in a CUDA graph over >= 4x L2 of weight copies.
decode_real_layers: the same step with the real decoder layer's structure inside the one launch (the
          four RMSNorms with weights, residual adds, layer scalars, GeGLU on a paired gate|up weight;
          helios_b200.stack.DecoderStack, the same weight bytes), and its time relative to `value`'s step.
decode_verify: the MTP verify widths (M = 1, 2, 4, 8 tokens per step) through the decode plan: ms per
          step and tokens/s, and per layer the step minus an LM-head-only plan of the same width over
          the layers (BASELINE config 2 through the plan), max over ranks.
cpu_baseline: the CPU oracle (fp32 accumulation, OpenMP on every host core) on a bounded sample
          (layer 0's seven projections at M = 1), rank 0 at N = 1 only.
prefill: BASELINE config 5 -- a 16384-token prompt as 8 chunks of 2048 tokens through all 48
          layers on the tcgen05 GEMM, then the LM head on the final row (each chunk its own seeded
          input); total ms and whole-job TFLOP/s, max over ranks; at N > 1 also the time of the
          chunk's 96 o/down allreduces run alone (same sizes, same collective), for the split of a
          chunk into GEMM and allreduce time.
parity: after every timed region, one decode step of a plan with per-layer output buffers (the
          same kernel and dataflow) is checked phase by phase against the CPU oracle on the GPU's
          own inputs (max excess over the bf16 rounding <= 1e-2 * rms for all 193 phases; the
          token is the argmax of the kernel's own softcapped logits and the oracle's up to a tie),
          plus the divergence of the oracle's own chained step. The oracle is only the checker
          here (tests/stack_parity.py); nothing it computes is timed or reported as a speed.
--impl reference: MLX (the reference's library) is absent, so the reference arm times the CPU
          restatement of the reference's CPU quantized_matmul (oracle/, kind "port") on the same
          metric with all host threads; ranks other than 0 exit without work.
--trace: after the timed regions, one decode step with the plan's tracing build (globaltimer stamps
          per CTA and phase) summarised per phase kind on rank 0 (the line's "trace" field, and
          "decode_real_layers.trace" for the real-layer step).
--case NAME: one small kernel case for an ncu capture (one GPU, a few GB at most; see CASES),
          printing its CUDA-event time per launch.
"""
from __future__ import annotations

import argparse
import csv
import io
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "4-bit qmatmul HBM GB/s (M=1), decode tok/s, prefill TFLOP/s at 1/2/4/8 B200"
WORKLOAD = ("decode step, batch 1: 48 layers x {q|k|v, o, gate|up, down} 4-bit g64 + tied LM head "
            "262144x3840 with softcap+argmax (BASELINE config 4)")


# Small self-contained cases for ncu captures (one GPU, a few GB at most): seeded weights (several
# copies where one matrix is smaller than L2, so consecutive launches read cold data), a few warm-up
# launches, then --launches timed ones; prints the CUDA-event time per launch.
CASES = {
    "gemv": dict(N=30720, K=3840, M=1, copies=4),      # fused gate|up decode GEMV, M = 1
    "gemv2": dict(N=30720, K=3840, M=2, copies=4),
    "gemv4": dict(N=30720, K=3840, M=4, copies=4),
    "gemv8": dict(N=30720, K=3840, M=8, copies=4),     # MTP verify width
    "up1": dict(N=15360, K=3840, M=1, copies=8),
    "down8": dict(N=3840, K=15360, M=8, copies=4),
    "lmhead": dict(N=262144, K=3840, M=1, copies=1),   # LM head + softcap + argmax
    "gemm": dict(N=8192, K=3840, M=2048, copies=1),    # prefill GEMM, q|k|v at 2048 tokens
    "gemm_kv": dict(N=2048, K=3840, M=2048, copies=1),     # 64 tiles: split-K in two
    "gemm_tp8": dict(N=1024, K=3840, M=2048, copies=1),    # a q|k|v shard at 8 ranks: split-K in four
    "dequant": dict(N=15360, K=3840, M=0, copies=1),   # bit-exact dequantize
    "decode": dict(layers=2),                          # persistent decode step, 2 full layers + LM head
    "decode_lm": dict(layers=0),                       # the same kernel, LM-head phase alone
}


def profile_case(a):
    import torch

    from helios_b200 import _lib
    from helios_b200.quantized import (QuantizedWeight, dequantize, lm_head_argmax, quantized_matmul, synth_matrix,
                                       synth_normal)
    from helios_b200.stack import StackConfig, SyntheticStack, activation_seed, matrix_seed
    _lib.load()
    torch.cuda.set_device(0)
    c = CASES[a.case]
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if a.case.startswith("decode"):
        cfg = StackConfig(layers=c["layers"])
        st = SyntheticStack(cfg, max_tokens=1)
        st.build_plan(1)
        h = synth_normal(activation_seed(0), (1, cfg.hidden))
        for _ in range(a.warmup):
            st.decode(h)
        torch.cuda.synchronize()
        e0.record()
        for _ in range(a.launches):
            st.decode(h)
        e1.record()
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) * 1e3 / a.launches
        wbytes = cfg.weight_bytes()
        print(json.dumps({"case": a.case, "us_per_launch": round(us, 3), "weight_bytes": wbytes,
                          "weight_GBps": round(wbytes / us / 1e3, 1)}))
        st.free()
        return
    ws = []
    for i in range(c["copies"]):
        w, s, b = synth_matrix(matrix_seed(i, "gate"), c["N"], c["K"])
        ws.append(QuantizedWeight.from_mlx(w, s, b))
        del w, s, b
    M = max(c["M"], 1)
    x = synth_normal(activation_seed(0), (M, c["K"]))
    y = torch.empty((M, c["N"]), dtype=torch.bfloat16, device="cuda")

    def run(i):
        q = ws[i % len(ws)]
        if a.case == "lmhead":
            lm_head_argmax(x, q, softcap=30.0, rms_scale=True)
        elif a.case == "dequant":
            dequantize(q)
        else:
            quantized_matmul(x, q, rms_scale=True, out=y)

    for i in range(a.warmup):
        run(i)
    torch.cuda.synchronize()
    e0.record()
    for i in range(a.launches):
        run(i)
    e1.record()
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / a.launches
    wbytes = c["N"] * c["K"] * 9 // 16
    out = {"case": a.case, "us_per_launch": round(us, 3), "weight_bytes": wbytes,
           "weight_GBps": round(wbytes / us / 1e3, 1)}
    if a.case.startswith("gemm"):
        out["TFLOPs"] = round(2 * c["M"] * c["N"] * c["K"] / us / 1e6, 1)
    print(json.dumps(out))


# words per CTA and phase of a decode-plan trace (g4q_decode_plan_trace): entry, x's producers done,
# x staged, then the end of each of the kernel's 16 warps' units
TRACE_WORDS = 3 + 16


def trace_summary(tr, layers: int) -> dict:
    """Per phase kind (q|k|v, o, gate|up, down; medians over the layers) of one traced step, in us:
    stage = x's producers done -> x staged (median CTA), compute = x staged -> the CTA's last warp
    done (median and slowest CTA), spread = slowest CTA's end - median CTA's end, lag = the previous
    phase's slowest CTA end -> this phase's median CTA staged, duration = slowest-CTA end to end."""
    import numpy as np

    t = tr.astype(np.int64)
    t = t - t[:, 0, 0].min()
    entry, prod, staged, wend = t[:, :, 0], t[:, :, 1], t[:, :, 2], t[:, :, 3:]
    cend = wend.max(axis=2)
    last_end = cend.max(axis=0)
    kinds = {"qkv": [], "o": [], "gu": [], "down": []}
    names = list(kinds)
    for p in range(1, 4 * layers):
        kinds[names[p % 4]].append([
            np.median(staged[:, p] - prod[:, p]), np.median(cend[:, p] - staged[:, p]),
            (cend[:, p] - staged[:, p]).max(), last_end[p] - np.median(cend[:, p]),
            np.median(staged[:, p]) - last_end[p - 1], last_end[p] - last_end[p - 1]])
    out = {"step_us": round(float(last_end[-1]) / 1e3, 1), "per_layer_us": 0.0,
           "columns": ["stage", "compute_med", "compute_max", "end_spread", "lag", "duration"]}
    for k, v in kinds.items():
        m = np.median(np.array(v), axis=0) / 1e3
        out[k] = [round(float(x), 2) for x in m]
        out["per_layer_us"] += float(m[5])
    out["per_layer_us"] = round(out["per_layer_us"], 2)
    p = 4 * layers
    out["lm"] = [round(float(x) / 1e3, 2) for x in (np.median(staged[:, p] - prod[:, p]),
                                                     np.median(cend[:, p] - staged[:, p]),
                                                     (cend[:, p] - staged[:, p]).max(),
                                                     last_end[p] - np.median(cend[:, p]),
                                                     np.median(staged[:, p]) - last_end[p - 1],
                                                     last_end[p] - last_end[p - 1])]
    return out


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=100)
    p.add_argument("--warmup", type=int, default=10)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--layers", type=int, default=48)
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-qmatmul", action="store_true", help="skip the standalone matmul section (configs 1 and 2)")
    p.add_argument("--prefill-tokens", type=int, default=2048, help="chunk size of the prefill measurement (0: skip)")
    p.add_argument("--prefill-chunks", type=int, default=8, help="chunks of the long prompt (config 5: 8 x 2048)")
    p.add_argument("--no-parity", action="store_true", help="skip the per-phase oracle check after timing")
    p.add_argument("--case", choices=sorted(CASES), help="run one small ncu case instead of the benchmark")
    p.add_argument("--launches", type=int, default=6, help="timed launches of --case")
    p.add_argument("--no-real-layers", action="store_true",
                   help="skip the step with the real decoder layer's norms, residuals and GeGLU in the plan")
    p.add_argument("--trace", action="store_true",
                   help="after timing, trace one decode step per phase and report a summary (profiling aid)")
    p.add_argument("--verify-steps", type=int, default=30,
                   help="timed steps per MTP-verify width through the plan (0: skip that section)")
    return p.parse_args()


def sustained_tflops() -> float:
    f = ROOT / "MEASURED_PEAKS.json"
    if f.exists():
        d = json.loads(f.read_text())
        return float(d.get("bf16_tflops_sustained", d["bf16_tflops"]))
    return 1400.0


def measured_peaks():
    f = ROOT / "MEASURED_PEAKS.json"
    if f.exists():
        d = json.loads(f.read_text())
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


class Clocks:
    """nvidia-smi sampling (200 ms) while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.idx), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (FileNotFoundError, OSError):
            self.proc = None
        time.sleep(0.3)

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.3)
        self.proc.terminate()
        out, _ = self.proc.communicate(timeout=10)
        rows = [r for r in csv.reader(io.StringIO(out)) if len(r) >= 9]
        sm = [float(r[1]) for r in rows if r[1].strip().replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].strip().replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].strip() == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


def cpu_baseline(seconds: float = 10.0):
    """Oracle qmm (fp32 accumulate, OpenMP, every host core) over layer 0's seven projections, M = 1."""
    from oracle import affine as A
    shapes = A.stack_shapes()
    mats = []
    for name in ("q", "k", "v", "o", "gate", "up", "down"):
        N, K = shapes[name]
        mats.append((A.synth_matrix(A.matrix_seed(0, A.PROJ_IDS[name]), N, K), K))
    xs = {K: A.synth_normal_bf16(A.activation_seed(0), K).reshape(1, K) for _, K in mats}
    nbytes = sum(m[0][0].nbytes + m[0][1].nbytes + m[0][2].nbytes for m in mats)
    cores = len(os.sched_getaffinity(0))
    reps, t0 = 0, time.perf_counter()
    while True:
        for (w, s, b), K in mats:
            A.qmm_f32(xs[K], w, s, b, threads=cores)
        reps += 1
        el = time.perf_counter() - t0
        if el >= seconds or reps >= 10000:
            break
    return {"value": round(nbytes * reps / el / 1e9, 3), "unit": "GB/s", "cores": cores, "kind": "port",
            "sample": f"layer 0's 7 projections at M=1 ({nbytes} B of packed weights+scales+biases) x {reps} passes "
                      f"in {el:.1f} s, oracle/g4q_oracle.c g4o_qmm_f32 (fp32 accumulate, OpenMP {cores} threads)"}


def run_reference(args, rank):
    if rank != 0:
        return
    from oracle import affine as A
    shapes = A.stack_shapes()
    mats = []
    for name in ("q", "k", "v", "o", "gate", "up", "down"):
        N, K = shapes[name]
        mats.append((A.synth_matrix(A.matrix_seed(0, A.PROJ_IDS[name]), N, K), K))
    xs = {K: A.synth_normal_bf16(A.activation_seed(0), K).reshape(1, K) for _, K in mats}
    nbytes = sum(m[0][0].nbytes + m[0][1].nbytes + m[0][2].nbytes for m in mats)
    cores = len(os.sched_getaffinity(0))

    def step():
        for (w, s, b), K in mats:
            A.qmm_f32(xs[K], w, s, b, threads=cores)
    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    el = time.perf_counter() - t0
    gbs = nbytes * args.steps / el / 1e9
    line = {
        "metric": METRIC, "value": round(gbs, 3), "unit": "GB/s", "impl": "reference", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(el / args.steps * 1e3, 4),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": WORKLOAD, "sample": "layer 0's 7 projections per step (bounded CPU sample)",
                   "tp": args.gpus},
        "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": cores, "kind": "port",
                         "sample": f"layer 0's 7 projections at M=1 ({nbytes} B) per step; MLX absent, timed the "
                                   f"C restatement of its CPU quantized_matmul (oracle/g4q_oracle.c, fp32 "
                                   f"accumulate, OpenMP {cores} threads)"},
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


LAYER_SHAPES = [("q", 4096, 3840), ("k", 2048, 3840), ("v", 2048, 3840), ("o", 3840, 4096),
                ("gate", 15360, 3840), ("up", 15360, 3840), ("down", 3840, 15360)]


def qmatmul_section(dev, hbm_peak: float) -> dict:
    """BASELINE configs 1 and 2 on the standalone matmul entry point (the stream-K GEMV): the
    up_proj 15360x3840 at M = 1, and one layer's seven projections at M in {1, 2, 4, 8}. Launches
    run back to back in a CUDA graph over enough weight copies that each launch reads its weights
    from HBM (at least 4x the L2 size in distinct copies). GB/s = algorithmic bytes (0.5625 B per
    weight + x reads + y writes) / device time per launch."""
    import torch

    from helios_b200.quantized import QuantizedWeight, quantized_matmul, synth_matrix, synth_normal
    from helios_b200.stack import activation_seed, matrix_seed

    l2 = torch.cuda.get_device_properties(dev).L2_cache_size

    def alg_bytes(N, K, M):
        return N * K * 9 // 16 + M * K * 2 + M * N * 2

    def timed(calls, reps=20):
        # warm, capture the list of launches once, replay `reps` times between two events
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            for c in calls:
                c()
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for c in calls:
                c()
        for _ in range(3):
            g.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            g.replay()
        e1.record()
        torch.cuda.synchronize()
        del g
        return e0.elapsed_time(e1) * 1e3 / (reps * len(calls))   # us per launch

    out = {"method": "CUDA graph of back-to-back g4q_qmm launches (stream-K GEMV, programmatic dependent "
                     "launch) cycling over >= 4x L2 of distinct weight copies; bf16 out",
           "peak": hbm_peak}
    # config 1: up_proj at M = 1
    N, K = 15360, 3840
    w, s, b = synth_matrix(matrix_seed(0, "up"), N, K, device=dev)
    copies = max(4, -(-4 * l2 // alg_bytes(N, K, 0)))
    ws = [QuantizedWeight.from_mlx(w, s, b) for _ in range(copies)]
    del w, s, b
    x = synth_normal(activation_seed(7), (1, K), device=dev)
    y = torch.empty((1, N), dtype=torch.bfloat16, device=dev)
    us = timed([lambda qw=qw: quantized_matmul(x, qw, out=y) for qw in ws])
    gbs = alg_bytes(N, K, 1) / (us * 1e-6) / 1e9
    out["config1_up_m1"] = {"shape": [N, K], "us": round(us, 2), "gbs": round(gbs, 1),
                            "frac": round(gbs / hbm_peak, 4), "weight_copies": copies}
    for qw in ws:
        qw.free()
    # config 2: one layer's seven projections at M in {1, 2, 4, 8}
    layer_bytes = sum(alg_bytes(n, k, 0) for _, n, k in LAYER_SHAPES)
    ncopy = max(2, -(-4 * l2 // layer_bytes))
    mats = []
    for c in range(ncopy):
        for name, n, k in LAYER_SHAPES:
            w, s, b = synth_matrix(matrix_seed(c, name), n, k, device=dev)
            mats.append((QuantizedWeight.from_mlx(w, s, b), n, k))
            del w, s, b
    layer = {}
    for M in (1, 2, 4, 8):
        xs = {k: synth_normal(activation_seed(M), (M, k), device=dev) for k in {k for _, _, k in LAYER_SHAPES}}
        ys = {n: torch.empty((M, n), dtype=torch.bfloat16, device=dev) for n in {n for _, n, _ in LAYER_SHAPES}}
        us = timed([lambda qw=qw, n=n, k=k: quantized_matmul(xs[k], qw, out=ys[n]) for qw, n, k in mats], reps=10)
        us_layer = us * len(LAYER_SHAPES)
        by = sum(alg_bytes(n, k, M) for _, n, k in LAYER_SHAPES)
        gbs = by / (us_layer * 1e-6) / 1e9
        layer[str(M)] = {"us_per_layer": round(us_layer, 2), "gbs": round(gbs, 1), "frac": round(gbs / hbm_peak, 4)}
    out["config2_layer"] = layer
    out["config2_layer_copies"] = ncopy
    for qw, _, _ in mats:
        qw.free()
    return out


def main():
    args = parse()
    if args.case:
        profile_case(args)
        return
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank)
        return

    import torch
    import torch.distributed as dist

    from helios_b200 import _lib
    from helios_b200.quantized import PHASE_ARGMAX, QMM_RMS_SCALE, DecodePlan, synth_normal
    from helios_b200.stack import StackConfig, SyntheticStack, activation_seed, decode_keys

    _lib.load()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    group = None
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
        group = dist.group.WORLD
    if args.gpus != world:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE {world}")

    cfg = StackConfig(layers=args.layers)
    st = SyntheticStack(cfg, rank, world, group)
    h_static = synth_normal(activation_seed(0), (1, cfg.hidden), device=dev)
    h_host = torch.empty((1, cfg.hidden), dtype=torch.bfloat16, pin_memory=True)
    h_host.copy_(h_static)
    key_host = torch.empty(1, dtype=torch.int64, pin_memory=True)

    def barrier():
        if world > 1:
            dist.barrier()

    # the whole decode step is one persistent-kernel launch per GPU (decode plan; tensor-parallel
    # plans reduce o/down over NVLink inside the kernel). Captured once, replayed per token.
    st.build_plan(1)
    step = lambda: st.decode(h_static)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(2):
            step()
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        keys, _ = step()
    for _ in range(max(args.warmup, 3)):
        graph.replay()
    torch.cuda.synchronize()

    def over_ranks(v: float):
        """(max, min) of a per-rank value over the ranks."""
        if world == 1:
            return v, v
        t = torch.tensor([v, -v], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t[0].item()), -float(t[1].item())

    clocks = Clocks(local)
    if rank == 0:
        clocks.start()
    # ---- device-timed decode steps
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        graph.replay()
    e1.record()
    torch.cuda.synchronize()
    barrier()
    ms_max, ms_min = over_ranks(e0.elapsed_time(e1) / args.steps)
    ms = ms_max
    # ---- end to end through the public API, every step: the pinned host hidden state copied in,
    #      one g4q_decode_plan_run call (SyntheticStack.decode), the token key read back to the host
    barrier()
    torch.cuda.synchronize()
    e2, e3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e2.record()
    for _ in range(args.steps):
        h_static.copy_(h_host, non_blocking=True)
        k_dev, _ = st.decode(h_static)
        key_host.copy_(k_dev[:1], non_blocking=True)
    e3.record()
    torch.cuda.synchronize()
    barrier()
    ms_e2e = over_ranks(e2.elapsed_time(e3) / args.steps)[0]
    clk = clocks.stop() if rank == 0 else None
    tok, _ = decode_keys(key_host)
    del graph

    # ---- MTP verify widths through the plan (decode_block_logits: M tokens per step, one launch) and
    #      BASELINE config 2 through the plan: per layer, the step minus an LM-head-only plan of the
    #      same width, over the layers
    verify = None
    if args.verify_steps > 0:
        verify = {"method": "CUDA graph of one plan run per step, CUDA events, max over ranks; per layer = "
                            "(step - LM-head-only plan) / layers"}
        for M in (1, 2, 4, 8):
            hM = synth_normal(activation_seed(M), (M, cfg.hidden), device=dev)
            xl = torch.zeros((M, cfg.hidden), dtype=torch.bfloat16, device=dev)
            lm_plan = DecodePlan([(st.lm, xl, None, QMM_RMS_SCALE | PHASE_ARGMAX)], M, rank=st.rank,
                                 n_ranks=st.size, group=st.group)
            st.build_plan(M)
            runs = {"step": lambda: st.decode(hM),
                    "lm": lambda: lm_plan.run(M, eps=cfg.eps, softcap=cfg.softcap, row_offset=st.v_rows[0],
                                              tokens=st.tokens[:M], values=st.values[:M], keys=st.keys[:M])}
            t = {}
            for name, fn in runs.items():
                s2 = torch.cuda.Stream()
                s2.wait_stream(torch.cuda.current_stream())
                with torch.cuda.stream(s2):
                    fn()
                torch.cuda.current_stream().wait_stream(s2)
                torch.cuda.synchronize()
                g2 = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g2):
                    fn()
                for _ in range(3):
                    g2.replay()
                barrier()
                torch.cuda.synchronize()
                f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                f0.record()
                for _ in range(args.verify_steps):
                    g2.replay()
                f1.record()
                torch.cuda.synchronize()
                barrier()
                t[name] = over_ranks(f0.elapsed_time(f1) / args.verify_steps)[0]
                del g2
            assert _lib.device_error() == 0
            lay_us = (t["step"] - t["lm"]) * 1e3 / cfg.layers
            verify[str(M)] = {"ms_per_step": round(t["step"], 5), "tok_s": round(M * 1e3 / t["step"], 1),
                              "weight_gbs": round(st.local_weight_bytes() * world / (t["step"] * 1e-3) / 1e9, 1),
                              "lm_head_only_us": round(t["lm"] * 1e3, 2), "us_per_layer": round(lay_us, 2)}
            lm_plan.free()
        st.plan.free()
        st.plan = None

    # ---- the real decoder layer's structure in the same single-launch step: input / post-attention /
    #      pre-FF / post-FF RMSNorms with their weights, residual adds, layer scalars and the GeGLU on a
    #      paired gate|up weight, all inside the decode kernel (DecoderStack: same weight bytes)
    real = None
    if not args.no_real_layers:
        from helios_b200.stack import DecoderStack
        ds = DecoderStack(cfg, rank, world, group, max_tokens=1)
        ds.build_plan(1)
        rstep = lambda: ds.decode(h_static)
        s3 = torch.cuda.Stream()
        s3.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s3):
            rstep()
        torch.cuda.current_stream().wait_stream(s3)
        torch.cuda.synchronize()
        g3 = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g3):
            rstep()
        for _ in range(max(args.warmup, 3)):
            g3.replay()
        barrier()
        torch.cuda.synchronize()
        f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        f0.record()
        for _ in range(args.steps):
            g3.replay()
        f1.record()
        torch.cuda.synchronize()
        barrier()
        ms_real = over_ranks(f0.elapsed_time(f1) / args.steps)[0]
        del g3
        assert _lib.device_error() == 0
        real = {"workload": "48 real-structure layers (norm weights, residual stream, layer scalars, GeGLU "
                            "phase) + final norm + LM head, one plan launch per step",
                "ms_per_step": round(ms_real, 5), "tok_s": round(1e3 / ms_real, 1),
                "weight_gbs": round(ds.local_weight_bytes() * world / (ms_real * 1e-3) / 1e9, 1),
                "vs_synthetic_step": round(ms_real / ms, 4), "token": decode_keys(ds.keys[:1])[0][0]}
        if args.trace:   # the same per-phase timeline summary as the linears-only step's `trace`
            buf = ds.plan.trace(True)
            for _ in range(3):
                ds.decode(h_static)
            torch.cuda.synchronize()
            barrier()
            ds.decode(h_static)
            torch.cuda.synchronize()
            assert _lib.device_error() == 0
            n_ph = 4 * cfg.layers + 1
            rtr = buf.cpu().view(-1, n_ph, TRACE_WORDS)
            ds.plan.trace(False)
            if rank == 0:
                real["trace"] = trace_summary(rtr.numpy(), cfg.layers)
        ds.free()

    # ---- per-phase timeline of one step (the plan's tracing build: globaltimer stamps per CTA and
    #      phase), summarised per phase kind on rank 0; a profiling aid, after the timed regions
    trace = None
    if args.trace:
        st.build_plan(1)
        buf = st.plan.trace(True)
        for _ in range(3):
            st.decode(h_static)
        torch.cuda.synchronize()
        barrier()
        st.decode(h_static)
        torch.cuda.synchronize()
        assert _lib.device_error() == 0
        n_ph = 4 * cfg.layers + 1
        tr = buf.cpu().view(-1, n_ph, TRACE_WORDS)
        st.plan.trace(False)
        st.plan.free()
        st.plan = None
        if rank == 0:
            trace = trace_summary(tr.numpy(), cfg.layers)

    # ---- chunked prefill: a 16384-token prompt as 8 chunks of 2048 tokens, each
    #      chunk through all layers on the tcgen05 GEMM path; the LM head on the final chunk's last
    #      row only. One chunk is captured in a CUDA graph (with the NCCL allreduces at N > 1) and
    #      replayed per chunk after a device copy of that chunk's seeded input; whole-job TFLOP/s.
    prefill = None
    if args.prefill_tokens > 0 and args.prefill_chunks > 0:
        P, C = args.prefill_tokens, args.prefill_chunks
        inputs = [synth_normal(activation_seed(1 + c), (P, cfg.hidden), device=dev) for c in range(C)]
        hp = torch.empty((P, cfg.hidden), dtype=torch.bfloat16, device=dev)
        hp.copy_(inputs[0])
        ps = torch.cuda.Stream()
        ps.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(ps):
            _, hlast = st.prefill(hp, head=False)
            st.head(hlast[P - 1:P])
        torch.cuda.current_stream().wait_stream(ps)
        torch.cuda.synchronize()
        g_chunk, g_head = torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph()
        with torch.cuda.graph(g_chunk):
            _, hlast = st.prefill(hp, head=False)
        with torch.cuda.graph(g_head):
            pkey, _ = st.head(hlast[P - 1:P])

        def prompt():
            for c in range(C):
                hp.copy_(inputs[c])
                g_chunk.replay()
            g_head.replay()

        prompt()   # warm-up run
        torch.cuda.synchronize()
        barrier()
        reps = 2
        p0, p1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        p0.record()
        for _ in range(reps):
            prompt()
        p1.record()
        torch.cuda.synchronize()
        barrier()
        total_ms = over_ranks(p0.elapsed_time(p1) / reps)[0]
        del g_chunk, g_head
        _, tf_burst, _ = measured_peaks()
        tf_sus = sustained_tflops()
        flops = st.cfg.flops_per_token() * P * C + 2 * cfg.vocab * cfg.hidden
        tflops = flops / (total_ms * 1e-3) / 1e12
        prefill = {"tokens": P * C, "chunk_tokens": P, "chunks": C, "layers": cfg.layers, "total_ms": round(total_ms, 3),
                   "ms_per_chunk": round(total_ms / C, 3), "flops": flops, "tflops": round(tflops, 1),
                   "unit": "TFLOP/s", "peak_sustained": round(tf_sus * world, 1),
                   "frac_of_sustained": round(tflops / (tf_sus * world), 4),
                   "peak_burst": round(tf_burst * world, 1), "frac_of_burst": round(tflops / (tf_burst * world), 4),
                   "timing": f"{reps} runs of the whole prompt after one warm-up run, CUDA events, max over ranks",
                   "path": "per chunk a CUDA graph: tcgen05 dequant-GEMM for every projection"
                           + (", NCCL allreduce of fp32 partials after o/down" if world > 1 else "")
                           + "; the LM head on the final row",
                   "gpu_launches_per_chunk": 6 * cfg.layers}   # q|k|v, gate|up: RMS rows + GEMM
        if world > 1:
            # the chunk's 96 o/down collectives alone (fp32 partials -> summed bf16 rows on every rank):
            # same sizes, same calls, captured the same way
            part = torch.zeros((P, cfg.hidden), dtype=torch.float32, device=dev)
            summed = torch.empty((P, cfg.hidden), dtype=torch.bfloat16, device=dev)
            ps.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(ps):
                st.sum_partials(part, summed)
            torch.cuda.current_stream().wait_stream(ps)
            torch.cuda.synchronize()
            g_ar = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g_ar):
                for _ in range(2 * cfg.layers):
                    st.sum_partials(part, summed)
            g_ar.replay()
            torch.cuda.synchronize()
            barrier()
            p0.record()
            g_ar.replay()
            p1.record()
            torch.cuda.synchronize()
            barrier()
            ar_ms = over_ranks(p0.elapsed_time(p1))[0]
            del g_ar
            prefill["allreduce_ms_per_chunk_alone"] = round(ar_ms, 3)
            prefill["allreduce_bytes_each"] = P * cfg.hidden * 4
            prefill["allreduce"] = "NCCL allreduce of the fp32 partials, then a cast to bf16"
        del inputs, hp

    hbm_peak, tf_peak, peak_kind = measured_peaks()
    # the dominant (only) kernel is the persistent decode kernel: one launch per step per rank
    kname = "decode_kernel (persistent: 48x{q|k|v, o, gate|up, down} + LM head, one launch per rank)"
    alg_bytes = st.local_weight_bytes() + 2 * cfg.hidden * 2 * (4 * cfg.layers + 1)
    launch_us = ms * 1e3
    traffic_file = ROOT / "profiles" / ("decode_kernel_traffic.json" if world == 1 else f"decode_kernel_tp{world}_traffic.json")
    achieved = alg_bytes / (launch_us * 1e-6) / 1e9
    traffic = None
    if traffic_file.exists():
        traffic = json.loads(traffic_file.read_text()).get("dram_bytes_per_launch")

    qmm = None
    if world == 1 and not args.no_qmatmul:
        qmm = qmatmul_section(dev, hbm_peak)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline()

    # ---- parity (after every timed region): one step of a plan with per-layer outputs, every phase
    #      checked on its own GPU input against the CPU oracle on rank 0
    parity = None
    if not args.no_parity:
        st.build_plan(1, keep_layers=True)
        logits = torch.empty((1, st.v_rows[1] - st.v_rows[0]), dtype=torch.bfloat16, device=dev)
        pk, _ = st.decode(h_static, logits=logits)
        torch.cuda.synchronize()
        perr = _lib.device_error()
        outs, lg = st.gather_layer_outputs(1, logits)
        if rank == 0:
            sys.path.insert(0, str(ROOT / "tests"))
            from oracle import affine as A
            from stack_parity import check_decode_step
            t_p, v_p = decode_keys(pk)
            h0 = h_static.view(torch.int16).cpu().numpy().view("uint16")
            t0 = time.perf_counter()
            parity = check_decode_step(A.stack_shapes(cfg.hidden, cfg.q_out, cfg.kv_out, cfg.inter, cfg.vocab),
                                       cfg.layers, h0, outs, t_p, v_p, logits=lg, softcap=cfg.softcap, eps=cfg.eps)
            parity["device_error"] = perr
            parity["token_equals_timed_step"] = t_p[0] == tok[0]
            parity["checker"] = (f"tests/stack_parity.py on the CPU oracle, {time.perf_counter() - t0:.1f} s, "
                                 "after the timed regions")
        barrier()

    wbytes = cfg.weight_bytes()
    gbs = wbytes / (ms * 1e-3) / 1e9
    gbs_e2e = wbytes / (ms_e2e * 1e-3) / 1e9
    if rank == 0:
        line = {
            "metric": METRIC, "value": round(gbs, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms, 5), "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded splitmix64 weights/activations)",
            "config": {"workload": WORKLOAD, "tokens_per_step": 1, "layers": cfg.layers,
                       "parallelism": f"tp{world}" if world > 1 else "single", "weight_bytes_per_step": wbytes,
                       "l2": "inputs larger than L2: 6.6 GB of weights streamed per step, no flush"},
            "decode_tok_s": round(1e3 / ms, 2),
            "decode_tok_s_e2e": round(1e3 / ms_e2e, 2),
            "ms_per_step_over_ranks": {"max": round(ms_max, 5), "min": round(ms_min, 5)},
            "e2e": {"value": round(gbs_e2e, 2), "unit": "GB/s", "h2d_bytes_per_step": cfg.hidden * 2,
                    "d2h_bytes_per_step": 8,
                    "path": "per step: pinned host hidden -> device, g4q_decode_plan_run (one C-ABI call), "
                            "token key -> pinned host"},
            "roofline": {"kernel": kname, "bound": "hbm", "achieved": round(achieved, 1),
                         "peak": hbm_peak, "unit": "GB/s", "frac": round(achieved / hbm_peak, 4),
                         "peak_kind": f"{peak_kind} hbm_gbs", "traffic": traffic,
                         "alg_bytes_per_launch": alg_bytes, "avg_launch_us": round(launch_us, 3)},
            "gpu_launches": 2 * args.steps,
            "clocks": clk,
            "last_token": tok[0],
        }
        if parity is not None:
            line["parity"] = parity
        if cpu is not None:
            line["cpu_baseline"] = cpu
        if prefill is not None:
            line["prefill"] = prefill
        if verify is not None:
            line["decode_verify"] = verify
        if trace is not None:
            line["trace"] = trace
        if real is not None:
            line["decode_real_layers"] = real
        if qmm is not None:
            line["qmatmul"] = qmm
        print(json.dumps(line), flush=True)
    barrier()
    st.free()
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
