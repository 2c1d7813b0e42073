"""CPU: the benchmark's host-side pieces -- the per-phase trace summary and the reference arm's line."""
import importlib.util
import json
import os
import subprocess
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent.parent


def _bench():
    spec = importlib.util.spec_from_file_location("bench_module", ROOT / "bench.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_trace_summary_reads_the_stamps():
    """Known stamps in, known durations out: 4 CTAs, 2 layers + the LM head (9 phases), phase p starting
    at 10 us * p; every CTA's producers are done 0.1 us after entry and x is staged 0.2 us later; its
    warps end 2 us after staging, CTA 0's 1 us later than the others."""
    bench = _bench()
    C, layers = 4, 2
    n_ph = 4 * layers + 1
    tr = np.zeros((C, n_ph, bench.TRACE_WORDS), dtype=np.int64)
    for p in range(n_ph):
        t = 10_000 * p
        for c in range(C):
            tr[c, p, 0] = t
            tr[c, p, 1] = t + 100
            tr[c, p, 2] = t + 300
            tr[c, p, 3:] = t + 2300 + (1000 if c == 0 else 0)
    out = bench.trace_summary(tr, layers)
    want = [0.2, 2.0, 3.0, 1.0, 7.0, 10.0]   # stage, loop med / max, spread, lag, duration (us)
    for kind in ("qkv", "o", "gu", "down", "lm"):
        assert out[kind] == want, (kind, out[kind])
    assert out["per_layer_us"] == 40.0
    assert out["step_us"] == 83.3
    assert out["columns"] == ["stage", "compute_med", "compute_max", "end_spread", "lag", "duration"]


def test_reference_arm_prints_one_json_line(oracle):
    """`bench.py --impl reference` (the CPU restatement of the reference's quantized_matmul, timed on
    the host cores) prints the benchmark's JSON line with the reference arm's fields."""
    r = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--steps", "1",
                        "--warmup", "1"], capture_output=True, text=True, timeout=300, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, r.stdout[-2000:]
    line = json.loads(lines[0])
    assert line["impl"] == "reference"
    assert line["metric"] == _bench().METRIC and line["unit"] == "GB/s" and line["value"] > 0
    assert line["higher_is_better"] is True and line["n_gpus"] == 1
    assert line["cpu_baseline"]["kind"] in ("port", "reference") and line["cpu_baseline"]["cores"] >= 1
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["d2h_bytes_per_step"] == 0
    assert line["e2e"]["value"] == line["value"]


def test_reference_arm_other_ranks_exit_without_work():
    """Under torchrun only rank 0 runs and prints the reference arm; rank 1 of 2 exits 0 at once."""
    env = dict(os.environ, RANK="1", WORLD_SIZE="2", LOCAL_RANK="1")
    r = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--gpus", "2",
                        "--steps", "1", "--warmup", "1"], capture_output=True, text=True, timeout=120,
                       cwd=ROOT, env=env)
    assert r.returncode == 0, r.stderr[-2000:]
    assert not [ln for ln in r.stdout.splitlines() if ln.startswith("{")], r.stdout[-2000:]
