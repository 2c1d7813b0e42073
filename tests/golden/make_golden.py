"""Generates the known-answer fixtures in tests/golden/ for the affine quantized format.

The reference project holds no golden vectors for quantized_matmul/dequantize and MLX (the
library that implements them) is absent, so these vectors are computed here from the format
definition with EXACT rational arithmetic (fractions.Fraction), independent of the C oracle:

* deq_kat.json      -- (scale, q, bias) -> bf16 of chain R1 = RN(s*q + b) and R2 = RN(RN(s*q) + b),
                       hand-picked special cases (identity, halves, subnormals, signed zeros,
                       overflow, R1 != R2 ties) plus seeded random finite bf16 triples.
* small_matrix.npz  -- one seeded 32 x 128 matrix: MLX-layout words, scales, biases, both
                       dequantized bf16 matrices (exact), x [3, 128] and y = x . deq^T (exact,
                       as float64 of the exact rational) for chain R2; generator outputs by the
                       numpy restatement; the layout-v1 words by a direct loop over the layout
                       definition.
* softcap_kat.json  -- bf16 logit -> bf16 softcap (l/30 in fp32 -> bf16 -> tanh in double -> fp32
                       -> bf16 -> *30 in fp32 -> bf16) over a sweep of bf16 patterns.

Run: python tests/golden/make_golden.py   (CPU only; writes next to this file)
"""
from __future__ import annotations

import json
import math
import random
import sys
from fractions import Fraction
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))

from oracle import affine as A  # noqa: E402  (exact restatement + numpy generator only)


def f32(x: float) -> np.float32:
    return np.float32(x)


def bf(x: float) -> int:
    return int(A.f32_to_bf16(np.float32(x)))


def deq_cases():
    cases = []
    one, half, zero = bf(1.0), bf(0.5), 0x0000
    for q in range(16):
        cases.append((one, q, zero))                 # identity: w = q
        cases.append((half, q, bf(-4.0)))            # w = q/2 - 4
        cases.append((bf(0.0137), q, bf(-0.1094)))   # typical g64 scale/bias
    cases.append((bf(1.0078125), 15, bf(-14.0)))     # R1 = 1.1171875, R2 = 1.125
    cases.append((bf(1.0078125), 15, bf(-7.0)))
    cases.append((bf(3.0517578e-05), 13, bf(-0.000244)))
    for sub in (0x0001, 0x0040, 0x007F, 0x8001, 0x807F):       # subnormal scales
        for q in (0, 1, 7, 15):
            cases.append((sub, q, 0x0000))
            cases.append((sub, q, 0x0001))
            cases.append((sub, q, 0x8000))
    for q in (0, 3):
        cases.append((0x8000, q, 0x8000))            # -0 * q + -0 = -0
        cases.append((0x8000, q, 0x0000))            # -0 + +0 = +0
        cases.append((bf(-2.0), 0, 0x8000))          # -0 + -0 = -0
    cases.append((0x7F7F, 15, 0x0000))               # overflow to +inf
    cases.append((0xFF7F, 15, 0x0000))               # overflow to -inf
    cases.append((0x7F7F, 1, 0xFF7F))                # max + (-max) = +0
    cases.append((bf(1e30), 9, bf(1e-30)))           # huge exponent gap (sticky bit decides)
    cases.append((bf(1.0078125), 9, bf(1e-30)))
    cases.append((bf(1.0078125), 9, bf(-1e-30)))
    rng = random.Random(20260630)

    def rnd():
        while True:
            h = rng.getrandbits(16)
            if (h >> 7) & 0xFF != 0xFF:
                return h
    for _ in range(1200):
        cases.append((rnd(), rng.randrange(16), rnd()))
    for _ in range(800):   # realistic exponent range
        s = (rng.getrandbits(1) << 15) | (rng.randrange(112, 130) << 7) | rng.getrandbits(7)
        b = (rng.getrandbits(1) << 15) | (rng.randrange(112, 130) << 7) | rng.getrandbits(7)
        cases.append((s, rng.randrange(16), b))
    return cases


def layout_words(w: np.ndarray, N: int, K: int) -> np.ndarray:
    """Layout v1 straight from its definition (independent loop, not the C oracle)."""
    R, G = N // 16, K // 64
    out = np.zeros(G * R * 128, dtype=np.uint32)

    def q_at(n, k):
        return (int(w[n, k // 8]) >> (4 * (k % 8))) & 15
    for g in range(G):
        for r in range(R):
            for lane in range(32):
                gi, t = lane // 4, lane % 4
                for j in range(4):
                    k0 = 64 * g + 16 * j
                    n0, n1 = 16 * r + gi, 16 * r + gi + 8
                    slots = [(n0, k0 + 2 * t), (n1, k0 + 2 * t), (n0, k0 + 2 * t + 8), (n1, k0 + 2 * t + 8),
                             (n0, k0 + 2 * t + 1), (n1, k0 + 2 * t + 1), (n0, k0 + 2 * t + 9), (n1, k0 + 2 * t + 9)]
                    word = 0
                    for slot, (n, k) in enumerate(slots):
                        word |= q_at(n, k) << (4 * slot)
                    out[(g * R + r) * 128 + lane * 4 + j] = word
    return out


def softcap_ref(h: int, cap: float = 30.0) -> int:
    l = A.bf16_to_f32(np.uint16(h))
    d = np.float32(l) / np.float32(cap)
    db = A.bf16_to_f32(A.f32_to_bf16(d))
    t = np.float32(math.tanh(float(db)))
    tb = A.bf16_to_f32(A.f32_to_bf16(t))
    return int(A.f32_to_bf16(tb * np.float32(cap)))


def main():
    # 1. dequant known answers
    kat = []
    for s, q, b in deq_cases():
        kat.append({"scale": s, "q": q, "bias": b, "r1": A.deq_exact(s, q, b, A.CHAIN_R1),
                    "r2": A.deq_exact(s, q, b, A.CHAIN_R2)})
    (HERE / "deq_kat.json").write_text(json.dumps({"chain_r1": "bf16(s*q+b)", "chain_r2": "bf16(bf16(s*q)+b)",
                                                    "cases": kat}))

    # 2. small seeded matrix, everything exact
    N, K, M = 32, 128, 3
    seed = A.matrix_seed(1, 5)
    w, s, b = A.np_synth_matrix(seed, N, K)
    x = np.empty(M * K, dtype=np.uint16)
    idx = np.arange(M * K, dtype=np.uint64)
    x[:] = A.f32_to_bf16(A.np_normal(A.activation_seed(7), idx))
    x = x.reshape(M, K)
    deq = {}
    for name, chain in (("deq_r1", A.CHAIN_R1), ("deq_r2", A.CHAIN_R2)):
        d = np.zeros((N, K), dtype=np.uint16)
        for n in range(N):
            for k in range(K):
                q = (int(w[n, k // 8]) >> (4 * (k % 8))) & 15
                d[n, k] = A.deq_exact(int(s[n, k // 64]), q, int(b[n, k // 64]), chain)
        deq[name] = d
    xv = [[A.bf16_value(int(v)) for v in row] for row in x]
    wv = [[A.bf16_value(int(v)) for v in row] for row in deq["deq_r2"]]
    y = np.zeros((M, N), dtype=np.float64)
    for m in range(M):
        for n in range(N):
            y[m, n] = float(sum((xv[m][k] * wv[n][k] for k in range(K)), Fraction(0)))
    rand_first = np.array([int(v) for v in A.np_rand(seed, np.arange(8, dtype=np.uint64))], dtype=np.uint64)
    np.savez_compressed(HERE / "small_matrix.npz", seed=np.uint64(seed), w=w, scales=s, biases=b, x=x,
                        deq_r1=deq["deq_r1"], deq_r2=deq["deq_r2"], y_r2=y, layout=layout_words(w, N, K),
                        rand_first=rand_first)

    # 3. softcap known answers (every 5th positive and negative finite pattern)
    pats = list(range(0, 0x7F80, 5)) + list(range(0x8000, 0xFF80, 5))
    (HERE / "softcap_kat.json").write_text(json.dumps({"cap": 30.0, "cases": [[h, softcap_ref(h)] for h in pats]}))
    print("wrote", [p.name for p in HERE.iterdir() if p.suffix in (".json", ".npz")])


if __name__ == "__main__":
    main()
