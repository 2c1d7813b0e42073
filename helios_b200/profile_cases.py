"""Small, self-contained kernel cases for ncu captures (one GPU, a few GB at most).

    python -m helios_b200.profile_cases gemv      # fused gate|up GEMV, 30720 x 3840, M = 1
    python -m helios_b200.profile_cases gemv8     # same at M = 8 (MTP verify width; also gemv2, gemv4)
    python -m helios_b200.profile_cases down8     # down 3840 x 15360 at M = 8
    python -m helios_b200.profile_cases lmhead    # LM head 262144 x 3840 + softcap + argmax, M = 1
    python -m helios_b200.profile_cases gemm      # prefill dequant-GEMM, q|k|v 8192 x 3840, M = 2048
    python -m helios_b200.profile_cases dequant   # bit-exact dequantize of 15360 x 3840
    python -m helios_b200.profile_cases decode    # persistent decode-step kernel, 2 full-size layers + LM head
    python -m helios_b200.profile_cases decode_lm # the same kernel with the LM-head phase alone (steady streaming)

Each case uploads seeded synthetic weights (several copies where the matrix is smaller than L2,
so consecutive launches read cold data), runs a few warm-up launches and then `--launches`
timed launches, and prints the CUDA-event average per launch.
"""
from __future__ import annotations

import argparse
import json

import torch

from .quantized import QuantizedWeight, dequantize, lm_head_argmax, quantized_matmul, synth_matrix, synth_normal
from .stack import activation_seed, matrix_seed

CASES = {
    "gemv": dict(N=30720, K=3840, M=1, copies=4),
    "gemv2": dict(N=30720, K=3840, M=2, copies=4),
    "gemv4": dict(N=30720, K=3840, M=4, copies=4),
    "gemv8": dict(N=30720, K=3840, M=8, copies=4),
    "down8": dict(N=3840, K=15360, M=8, copies=4),
    "lmhead": dict(N=262144, K=3840, M=1, copies=1),
    "gemm": dict(N=8192, K=3840, M=2048, copies=1),
    "gemm_kv": dict(N=2048, K=3840, M=2048, copies=1),     # 64 tiles: split-K in two
    "gemm_tp8": dict(N=1024, K=3840, M=2048, copies=1),    # a q|k|v shard at 8 ranks: split-K in four
    "dequant": dict(N=15360, K=3840, M=0, copies=1),
    "decode": dict(layers=2),
    "decode_lm": dict(layers=0),
}


def decode_case(a, c):
    """The single-launch decode plan of a 2-layer full-width stack (about 0.8 GB of weights)."""
    from .stack import StackConfig, SyntheticStack
    cfg = StackConfig(layers=c["layers"])
    st = SyntheticStack(cfg, max_tokens=1)
    st.build_plan(1)
    h = synth_normal(activation_seed(0), (1, cfg.hidden))
    for _ in range(a.warmup):
        st.decode(h)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
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


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("case", choices=sorted(CASES))
    ap.add_argument("--launches", type=int, default=6)
    ap.add_argument("--warmup", type=int, default=2)
    a = ap.parse_args()
    c = CASES[a.case]
    torch.cuda.set_device(0)
    if a.case.startswith("decode"):
        return decode_case(a, c)
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
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
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


if __name__ == "__main__":
    main()
