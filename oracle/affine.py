"""Python side of the CPU oracle for MLX's affine quantized format.

TEST INFRASTRUCTURE ONLY. Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s
CPU-baseline / reference arm import this module, as the checker or as the timed CPU
stand-in for MLX's CPU ``quantized_matmul``. The product (``helios_b200`` and
``libg4q.so``) never imports it.

Two independent restatements live here:

* ``lib()`` -- ctypes bindings to ``oracle/libg4q_oracle.so`` (the C restatement in
  ``g4q_oracle.c``), fast enough for full-size layers.
* ``deq_exact`` / ``bf16_round_exact`` -- exact rational arithmetic (``fractions``) of the
  same format definition, used to pin the C oracle on the known-answer vectors in
  ``tests/golden``; and ``np_rand`` / ``np_synth_matrix``, a numpy restatement of the
  seeded generator.

Reference behaviour restated (paths relative to the reference project):
``native/gemma4_mlx/src/native_model.cc:349-362`` (quantized_linear: affine
``quantized_matmul`` with transpose=true, then bf16), ``:364-376`` (quantized_embedding:
take + ``dequantize``), ``:1782-1795`` (tied LM head, bf16 ``tanh(l/30)*30`` softcap),
``:3825`` (argmax, first index wins). Parity with MLX itself is unpinned: MLX 0.31.2 is
absent and the reference holds no golden vectors for this path.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from fractions import Fraction
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "libg4q_oracle.so"

CHAIN_R1 = 1
CHAIN_R2 = 2
MASK64 = (1 << 64) - 1

_lib = None


def build() -> Path:
    """Compile the C oracle with oracle/Makefile (gcc, no GPU needed)."""
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            build()
        L = ctypes.CDLL(str(LIB_PATH))
        P = ctypes.c_void_p
        i64, i32, u64 = ctypes.c_int64, ctypes.c_int, ctypes.c_uint64
        L.g4o_set_threads.restype = None
        L.g4o_set_threads.argtypes = [i32]
        L.g4o_rand.restype = u64
        L.g4o_rand.argtypes = [u64, u64]
        L.g4o_matrix_seed.restype = u64
        L.g4o_matrix_seed.argtypes = [i32, i32]
        L.g4o_activation_seed.restype = u64
        L.g4o_activation_seed.argtypes = [i32]
        L.g4o_synth_matrix.argtypes = [u64, i64, i64, i32, i32, P, P, P]
        L.g4o_synth_normal_bf16.argtypes = [u64, i64, P]
        L.g4o_deq1.restype = ctypes.c_uint16
        L.g4o_deq1.argtypes = [ctypes.c_uint16, ctypes.c_uint32, ctypes.c_uint16, i32]
        L.g4o_dequantize.argtypes = [P, P, P, i64, i64, i32, i32, i32, P]
        L.g4o_dequantize_rows.argtypes = [P, P, P, i64, i64, i32, i32, i32, P, i64, P]
        L.g4o_qmm.argtypes = [P, i64, P, P, P, i64, i64, i32, i32, i32, P, P, P]
        L.g4o_qmm_f32.argtypes = [P, i64, P, P, P, i64, i64, i32, i32, i32, P]
        L.g4o_rms_scale.restype = ctypes.c_float
        L.g4o_rms_scale.argtypes = [P, i64, ctypes.c_float]
        L.g4o_tanh.restype = ctypes.c_float
        L.g4o_tanh.argtypes = [ctypes.c_float]
        L.g4o_softcap.restype = ctypes.c_uint16
        L.g4o_softcap.argtypes = [ctypes.c_uint16, ctypes.c_float]
        L.g4o_softcap_argmax.argtypes = [P, i64, ctypes.c_float, P, P]
        L.g4o_repack.argtypes = [P, P, P, i64, i64, P, P]
        L.g4o_unpack.argtypes = [P, P, i64, i64, P, P, P]
        _lib = L
    return _lib


def _p(a: np.ndarray):
    assert a.flags["C_CONTIGUOUS"], "oracle arrays must be C-contiguous"
    return ctypes.c_void_p(a.ctypes.data)


def _check(rc: int, what: str):
    if rc != 0:
        raise ValueError(f"oracle {what} rejected its arguments (rc={rc})")


# ----------------------------------------------------------------- bf16 helpers --
def bf16_to_f32(h: np.ndarray) -> np.ndarray:
    return (np.asarray(h, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16(f: np.ndarray) -> np.ndarray:
    arr = np.asarray(f, dtype=np.float32)
    u = np.atleast_1d(arr).view(np.uint32).astype(np.uint64)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
    return r.reshape(arr.shape)


# ----------------------------------------------------------------- generator --
def matrix_seed(layer: int, proj: int) -> int:
    return 0x48454C494F53 ^ (layer * 16 + proj)


def activation_seed(chunk: int) -> int:
    return 0x48454C494F53 ^ 0xF00 ^ chunk


def synth_matrix(seed: int, N: int, K: int, bits: int = 4, group_size: int = 64):
    w = np.empty((N, K * bits // 32), dtype=np.uint32)
    s = np.empty((N, K // group_size), dtype=np.uint16)
    b = np.empty((N, K // group_size), dtype=np.uint16)
    lib().g4o_synth_matrix(seed, N, K, bits, group_size, _p(w), _p(s), _p(b))
    return w, s, b


def synth_normal_bf16(seed: int, count: int) -> np.ndarray:
    out = np.empty(count, dtype=np.uint16)
    lib().g4o_synth_normal_bf16(seed, count, _p(out))
    return out


def np_rand(seed: int, index: np.ndarray) -> np.ndarray:
    """numpy restatement of the counter-based splitmix64 stream."""
    with np.errstate(over="ignore"):
        z = np.uint64(seed) + (np.asarray(index, dtype=np.uint64) + np.uint64(1)) * np.uint64(0x9E3779B97F4A7C15)
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
        return z ^ (z >> np.uint64(31))


def np_normal(seed: int, index: np.ndarray) -> np.ndarray:
    index = np.asarray(index, dtype=np.uint64)
    total = np.zeros(index.shape, dtype=np.int64)
    for j in range(3):
        r = np_rand(seed, np.uint64(3) * index + np.uint64(j))
        for sh in (0, 16, 32, 48):
            total += ((r >> np.uint64(sh)) & np.uint64(0xFFFF)).astype(np.int64)
    return (total - 393216).astype(np.float32) * np.float32(1.0 / 65536.0)


def np_synth_matrix(seed: int, N: int, K: int, bits: int = 4, group_size: int = 64):
    """Independent numpy restatement of g4o_synth_matrix (float32 ops, one rounding each)."""
    seed_w = int(np_rand(seed, np.array([1]))[0])
    seed_s = int(np_rand(seed, np.array([2]))[0])
    seed_b = int(np_rand(seed, np.array([3]))[0])
    nw = N * K * bits // 32
    w = (np_rand(seed_w, np.arange(nw, dtype=np.uint64)) >> np.uint64(32)).astype(np.uint32)
    G = N * (K // group_size)
    idx = np.arange(G, dtype=np.uint64)
    u = (np_rand(seed_s, idx) >> np.uint64(40)).astype(np.float32) * np.float32(5.9604644775390625e-8)
    sv = np.float32(0.002) + u * np.float32(0.018)
    s = f32_to_bf16(sv)
    t1 = np.float32(-8.0) * bf16_to_f32(s)
    t2 = np.float32(1e-3) * np_normal(seed_b, idx)
    b = f32_to_bf16(t1 + t2)
    return w.reshape(N, -1), s.reshape(N, -1), b.reshape(N, -1)


# ----------------------------------------------------------------- format (C) --
def deq1(scale: int, q: int, bias: int, chain: int = CHAIN_R2) -> int:
    return int(lib().g4o_deq1(scale, q, bias, chain))


def dequantize(w, s, b, bits: int = 4, group_size: int = 64, chain: int = CHAIN_R2) -> np.ndarray:
    N = w.shape[0]
    K = w.shape[1] * 32 // bits
    out = np.empty((N, K), dtype=np.uint16)
    _check(lib().g4o_dequantize(_p(w), _p(s), _p(b), N, K, bits, group_size, chain, _p(out)), "dequantize")
    return out


def dequantize_rows(w, s, b, ids, bits: int = 4, group_size: int = 64, chain: int = CHAIN_R2):
    N = w.shape[0]
    K = w.shape[1] * 32 // bits
    ids = np.ascontiguousarray(ids, dtype=np.int32)
    out = np.empty((ids.size, K), dtype=np.uint16)
    _check(lib().g4o_dequantize_rows(_p(w), _p(s), _p(b), N, K, bits, group_size, chain,
                                     _p(ids), ids.size, _p(out)), "dequantize_rows")
    return out


def qmm(x, w, s, b, bits: int = 4, group_size: int = 64, chain: int = CHAIN_R2, row_scale=None):
    """Returns (y_exact float64 [M,N], y_bf16 uint16 [M,N])."""
    x = np.ascontiguousarray(x, dtype=np.uint16)
    M, K = x.shape
    N = w.shape[0]
    assert w.shape[1] * 32 // bits == K
    ye = np.empty((M, N), dtype=np.float64)
    yb = np.empty((M, N), dtype=np.uint16)
    rs = None if row_scale is None else np.ascontiguousarray(row_scale, dtype=np.float32)
    _check(lib().g4o_qmm(_p(x), M, _p(w), _p(s), _p(b), N, K, bits, group_size, chain,
                         None if rs is None else _p(rs), _p(ye), _p(yb)), "qmm")
    return ye, yb


def set_threads(n: int) -> None:
    """OpenMP threads of the oracle's loops (n <= 0: the runtime's default)."""
    lib().g4o_set_threads(int(n))


def qmm_f32(x, w, s, b, group_size: int = 64, chain: int = CHAIN_R2, threads: int = 0):
    x = np.ascontiguousarray(x, dtype=np.uint16)
    M, K = x.shape
    N = w.shape[0]
    y = np.empty((M, N), dtype=np.uint16)
    _check(lib().g4o_qmm_f32(_p(x), M, _p(w), _p(s), _p(b), N, K, group_size, chain, threads, _p(y)),
           "qmm_f32")
    return y


def lora_scale_bf16(alpha: float, rank: int) -> float:
    """bf16(alpha / rank) as a float: the adapter scale (native_model.cc:3378) as model_scalar
    rounds it (:342-347), the fp32 quotient first."""
    q = np.float32(np.float32(alpha) / np.float32(rank))
    return float(bf16_to_f32(f32_to_bf16(q)))


def lora_delta(x, y_base, lora_a, lora_b, alpha: float):
    """add_lora_delta_if_active (native_model.cc:316-328) on a bf16 base output.

    x: bf16 bits [M, K]; y_base: bf16 bits [M, N]; lora_a: [rank, K]; lora_b: [N, rank] (both
    converted to fp32 as at :3419-3420). low = f32(x) @ A^T and delta = low @ B^T are accumulated in
    float64 and rounded once to fp32 (the fp32 matmul results), then delta * bf16(alpha/rank) in
    fp32, bf16(delta), and the bf16 add bf16(y_base + delta). Returns the bf16 bits [M, N]."""
    x = np.ascontiguousarray(x, dtype=np.uint16)
    a = np.asarray(lora_a, dtype=np.float32).astype(np.float64)
    b = np.asarray(lora_b, dtype=np.float32).astype(np.float64)
    rank = a.shape[0]
    low = (bf16_to_f32(x).astype(np.float64) @ a.T).astype(np.float32)
    mm = (low.astype(np.float64) @ b.T).astype(np.float32)
    delta = f32_to_bf16(mm * np.float32(lora_scale_bf16(alpha, rank)))
    out = bf16_to_f32(np.asarray(y_base, dtype=np.uint16)) + bf16_to_f32(delta)
    return f32_to_bf16(out.astype(np.float32))


def _rb(a) -> np.ndarray:
    """fp32 -> bf16 (round to nearest even) -> fp32."""
    return bf16_to_f32(f32_to_bf16(np.asarray(a, dtype=np.float32)))


def geglu(gate, up):
    """geglu (native_model.cc:378-386) on bf16 bits: the nine bf16 ops of the reference, each an
    fp32 operation on bf16 operands rounded to bf16, with the constants as model_scalar rounds them
    (bf16(0.044715), bf16(0.7978845608028654), 0.5, 1.0); gate^3 as g*g*g (exact in fp32)."""
    g = bf16_to_f32(gate)
    u = bf16_to_f32(up)
    kc = np.float32(_rb(np.float32(0.044715)))
    ka = np.float32(_rb(np.float32(0.7978845608028654)))
    g3 = _rb(g * g * g)
    t1 = _rb(kc * g3)
    t2 = _rb(g + t1)
    t3 = _rb(ka * t2)
    t4 = _rb(np.tanh(t3))
    t5 = _rb(np.float32(1.0) + t4)
    t6 = _rb(np.float32(0.5) * g)
    t7 = _rb(t6 * t5)
    return f32_to_bf16(t7 * u)


def rms_norm(x, weight=None, eps: float = 1e-6):
    """model_dtype(fast::rms_norm(x, weight, eps)) on bf16 bits [..., K]: mean(x^2) accumulated in
    float64 and rounded to fp32, inv = 1/sqrt(mean + eps) correctly rounded to fp32, then
    bf16(weight * bf16(x * inv)) (the normalized value rounded to the input dtype before the weight
    product, as MLX's fast::rms_norm does)."""
    xf = bf16_to_f32(x)
    m = np.float32((xf.astype(np.float64) ** 2).mean(axis=-1, keepdims=True))
    v = (m + np.float32(eps)).astype(np.float32)
    inv = (1.0 / np.sqrt(v.astype(np.float64))).astype(np.float32)
    y = _rb(xf * inv)
    if weight is None:
        return f32_to_bf16(y)
    return f32_to_bf16(bf16_to_f32(weight) * y)


def rms_norm_residual(x, weight, residual, layer_scalar=None, eps: float = 1e-6):
    """native_model.cc:954-968 on bf16 bits: n = rms_norm(x, weight); h = bf16(residual + n); then
    bf16(h * layer_scalar) when a scalar (bf16 bits) is given -- each op one bf16 rounding."""
    n = bf16_to_f32(rms_norm(x, weight, eps))
    h = _rb(bf16_to_f32(residual) + n)
    if layer_scalar is None:
        return f32_to_bf16(h)
    return f32_to_bf16(h * np.float32(bf16_to_f32(np.asarray([layer_scalar], np.uint16))[0]))


def rms_scale(x_row, eps: float = 1e-6) -> float:
    x_row = np.ascontiguousarray(x_row, dtype=np.uint16)
    return float(lib().g4o_rms_scale(_p(x_row), x_row.size, eps))


def tanh(x: float) -> float:
    return float(lib().g4o_tanh(x))


def softcap(logit_bits: int, cap: float = 30.0) -> int:
    return int(lib().g4o_softcap(logit_bits, cap))


def softcap_argmax(logits, cap: float = 30.0):
    logits = np.ascontiguousarray(logits, dtype=np.uint16).ravel()
    tok = np.zeros(1, dtype=np.int32)
    val = np.zeros(1, dtype=np.float32)
    _check(lib().g4o_softcap_argmax(_p(logits), logits.size, cap, _p(tok), _p(val)), "softcap_argmax")
    return int(tok[0]), float(val[0])


def repack(w, s, b):
    N = w.shape[0]
    K = w.shape[1] * 8
    packed = np.empty(N * K // 8, dtype=np.uint32)
    sb = np.empty(N * K // 64, dtype=np.uint32)
    _check(lib().g4o_repack(_p(w), _p(s), _p(b), N, K, _p(packed), _p(sb)), "repack")
    return packed, sb


def unpack(packed, sb, N: int, K: int):
    w = np.empty((N, K // 8), dtype=np.uint32)
    s = np.empty((N, K // 64), dtype=np.uint16)
    b = np.empty((N, K // 64), dtype=np.uint16)
    _check(lib().g4o_unpack(_p(packed), _p(sb), N, K, _p(w), _p(s), _p(b)), "unpack")
    return w, s, b


# ----------------------------------------------------------------- exact restatement --
def bf16_value(bits: int) -> Fraction:
    """Exact rational value of a finite bf16 bit pattern."""
    bits &= 0xFFFF
    sign = -1 if bits & 0x8000 else 1
    e = (bits >> 7) & 0xFF
    m = bits & 0x7F
    if e == 0xFF:
        raise ValueError("non-finite bf16")
    if e == 0:
        return sign * Fraction(m, 1) * Fraction(1, 2 ** 133)
    return sign * (Fraction(128 + m, 128)) * (Fraction(2) ** (e - 127))


def bf16_round_exact(v: Fraction, negative_zero: bool = False) -> int:
    """bf16 round-to-nearest-even of an exact rational (finite, may overflow to inf)."""
    if v == 0:
        return 0x8000 if negative_zero else 0x0000
    sign = 0x8000 if v < 0 else 0
    a = -v if v < 0 else v
    # binade: 2^e <= a < 2^(e+1)
    e = a.numerator.bit_length() - a.denominator.bit_length()
    if Fraction(2) ** e > a:
        e -= 1
    qexp = max(e - 7, -133)
    t = a / (Fraction(2) ** qexp)
    n = t.numerator // t.denominator
    frac = t - n
    if frac > Fraction(1, 2) or (frac == Fraction(1, 2) and n % 2 == 1):
        n += 1
    r = n * (Fraction(2) ** qexp)
    if r >= Fraction(2) ** 128:
        return sign | 0x7F80
    if r < Fraction(2) ** -126:          # subnormal: mantissa = r / 2^-133
        return sign | int(r * 2 ** 133)
    re = qexp + 7                         # binade of r (may have carried)
    mant = r / (Fraction(2) ** re)
    if mant >= 2:
        re += 1
        mant /= 2
    return sign | ((re + 127) << 7) | int((mant - 1) * 128)


def deq_exact(scale: int, q: int, bias: int, chain: int = CHAIN_R2) -> int:
    """The format definition in exact arithmetic: R1 = bf16(s*q + b), R2 = bf16(bf16(s*q) + b)."""
    s = bf16_value(scale)
    b = bf16_value(bias)
    # IEEE signs of zeros: s*q (q >= 0) is -0 exactly when it is zero and s is negative;
    # an exact-zero sum under round-to-nearest is -0 only when both addends are -0.
    prod_neg_zero = (s * q == 0) and bool(scale & 0x8000)
    bias_neg_zero = (b == 0) and bool(bias & 0x8000)
    if chain == CHAIN_R1:
        v = s * q + b
        return bf16_round_exact(v, negative_zero=(prod_neg_zero and bias_neg_zero))
    p_bits = bf16_round_exact(s * q, negative_zero=prod_neg_zero)
    if p_bits & 0x7FFF == 0x7F80:          # s*q overflowed: inf + finite bias stays inf
        return p_bits
    p = bf16_value(p_bits)
    v = p + b
    p_neg_zero = (p == 0) and bool(p_bits & 0x8000)
    return bf16_round_exact(v, negative_zero=(p_neg_zero and bias_neg_zero))


# ----------------------------------------------------------------- synthetic stack --
# Synthetic decoder stack of the benchmark (BASELINE config 4/5 shapes): per layer the
# seven 4-bit g64 projections, proj ids q0 k1 v2 o3 gate4 up5 down6, LM head id 7.
PROJ_IDS = {"q": 0, "k": 1, "v": 2, "o": 3, "gate": 4, "up": 5, "down": 6, "lm": 7}


def stack_shapes(hidden=3840, q_out=4096, kv_out=2048, inter=15360, vocab=262144):
    return {"q": (q_out, hidden), "k": (kv_out, hidden), "v": (kv_out, hidden),
            "o": (hidden, q_out), "gate": (inter, hidden), "up": (inter, hidden),
            "down": (hidden, inter), "lm": (vocab, hidden)}


def stack_matrix(layer: int, name: str, shapes):
    N, K = shapes[name]
    return synth_matrix(matrix_seed(0 if name == "lm" else layer, PROJ_IDS[name]), N, K)


def stack_forward(h0, n_layers: int, shapes, cap: float = 30.0, eps: float = 1e-6,
                  chain: int = CHAIN_R2, matrices=None):
    """Oracle of the synthetic linear stack (one decode step or one chunk of M rows).

    For each layer: a = rms(h); qkv = bf16(a * h.Wqkv^T); o = bf16(q.Wo^T);
    gu = bf16(rms(o) * o.Wgu^T); h = bf16(up.Wdown^T). Then logits = bf16(rms(h) * h.Wlm^T)
    and the token is argmax(softcap(logits)) per row. rms(v) = 1/sqrt(mean(v^2)+eps) per
    row, applied to the product (y = r * (x.W^T)).
    Returns dict with the final hidden (uint16), logits (uint16), tokens, values.
    """
    get = matrices if matrices is not None else (lambda l, n: stack_matrix(l, n, shapes))
    h = np.ascontiguousarray(h0, dtype=np.uint16)
    M = h.shape[0]
    for layer in range(n_layers):
        r = np.array([rms_scale(h[m], eps) for m in range(M)], dtype=np.float32)
        q = qmm(h, *get(layer, "q"), chain=chain, row_scale=r)[1]
        for name in ("k", "v"):
            qmm(h, *get(layer, name), chain=chain, row_scale=r)
        o = qmm(q, *get(layer, "o"), chain=chain)[1]
        r2 = np.array([rms_scale(o[m], eps) for m in range(M)], dtype=np.float32)
        qmm(o, *get(layer, "gate"), chain=chain, row_scale=r2)
        up = qmm(o, *get(layer, "up"), chain=chain, row_scale=r2)[1]
        h = qmm(up, *get(layer, "down"), chain=chain)[1]
    r3 = np.array([rms_scale(h[m], eps) for m in range(M)], dtype=np.float32)
    ye, logits = qmm(h, *get(0, "lm"), chain=chain, row_scale=r3)
    toks, vals = [], []
    for m in range(M):
        t, v = softcap_argmax(logits[m], cap)
        toks.append(t)
        vals.append(v)
    return {"hidden": h, "logits": logits, "logits_exact": ye, "tokens": toks, "values": vals}
