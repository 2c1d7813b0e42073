"""Pins the CPU oracle (oracle/g4q_oracle.c) to the known-answer fixtures in tests/golden.

The fixtures come from exact rational arithmetic of the format definition
(tests/golden/make_golden.py) because the reference holds no vectors for this path and MLX
is absent; see the oracle header for what that leaves unpinned.
"""
import json

import numpy as np
import pytest

from conftest import GOLDEN


def test_deq_known_answers_both_chains(oracle):
    kat = json.loads((GOLDEN / "deq_kat.json").read_text())["cases"]
    assert len(kat) > 2000
    bad = []
    for c in kat:
        for chain, key in ((oracle.CHAIN_R1, "r1"), (oracle.CHAIN_R2, "r2")):
            got = oracle.deq1(c["scale"], c["q"], c["bias"], chain)
            if got != c[key]:
                bad.append((c, key, hex(got)))
    assert not bad, bad[:5]


def test_r1_and_r2_really_differ_somewhere(oracle):
    kat = json.loads((GOLDEN / "deq_kat.json").read_text())["cases"]
    assert sum(c["r1"] != c["r2"] for c in kat) > 50


def test_exact_restatement_matches_itself_on_hand_cases(oracle):
    bf = lambda v: int(oracle.f32_to_bf16(np.float32(v)))
    s, b = bf(1.0078125), bf(-14.0)
    assert oracle.bf16_value(oracle.deq_exact(s, 15, b, oracle.CHAIN_R1)) == 1.1171875
    assert oracle.bf16_value(oracle.deq_exact(s, 15, b, oracle.CHAIN_R2)) == 1.125
    for q in range(16):
        assert oracle.bf16_value(oracle.deq_exact(bf(1.0), q, 0, oracle.CHAIN_R2)) == q


def test_generator_c_vs_numpy_and_fixture(oracle):
    z = np.load(GOLDEN / "small_matrix.npz")
    seed = int(z["seed"])
    w, s, b = oracle.synth_matrix(seed, 32, 128)
    assert (w == z["w"]).all() and (s == z["scales"]).all() and (b == z["biases"]).all()
    first = np.array([oracle.lib().g4o_rand(seed, i) for i in range(8)], dtype=np.uint64)
    assert (first == z["rand_first"]).all()
    for sd, (N, K) in ((oracle.matrix_seed(3, 4), (48, 256)), (99, (16, 64))):
        a = oracle.synth_matrix(sd, N, K)
        c = oracle.np_synth_matrix(sd, N, K)
        assert all((u == v).all() for u, v in zip(a, c))


def test_generator_distributions(oracle):
    w, s, b = oracle.synth_matrix(oracle.matrix_seed(0, 5), 256, 3840)
    sf, bfv = oracle.bf16_to_f32(s), oracle.bf16_to_f32(b)
    assert 0.00199 <= sf.min() and sf.max() <= 0.0201   # bf16 rounding of U(0.002, 0.02)
    resid = bfv + 8 * sf
    assert abs(resid.mean()) < 2e-4 and 0.5e-3 < resid.std() < 1.5e-3
    q = np.concatenate([(w >> (4 * j)) & 15 for j in range(8)]).ravel()
    counts = np.bincount(q, minlength=16)
    assert counts.min() > 0.9 * counts.mean()
    x = oracle.bf16_to_f32(oracle.synth_normal_bf16(oracle.activation_seed(0), 200000))
    assert abs(x.mean()) < 0.01 and abs(x.std() - 1) < 0.01


def test_dequantize_matrix_exact(oracle):
    z = np.load(GOLDEN / "small_matrix.npz")
    for name, chain in (("deq_r1", oracle.CHAIN_R1), ("deq_r2", oracle.CHAIN_R2)):
        d = oracle.dequantize(z["w"], z["scales"], z["biases"], chain=chain)
        assert (d == z[name]).all(), name


def test_dequantize_rows_and_bad_ids(oracle):
    z = np.load(GOLDEN / "small_matrix.npz")
    ids = np.array([31, 0, 7, 7], dtype=np.int32)
    d = oracle.dequantize_rows(z["w"], z["scales"], z["biases"], ids)
    assert (d == z["deq_r2"][ids]).all()
    with pytest.raises(ValueError):
        oracle.dequantize_rows(z["w"], z["scales"], z["biases"], np.array([32], dtype=np.int32))


def test_qmm_matches_exact_rational(oracle):
    z = np.load(GOLDEN / "small_matrix.npz")
    ye, yb = oracle.qmm(z["x"], z["w"], z["scales"], z["biases"])
    np.testing.assert_allclose(ye, z["y_r2"], rtol=1e-12, atol=1e-12)
    assert (yb == oracle.f32_to_bf16(z["y_r2"].astype(np.float32))).mean() > 0.95


def test_qmm_f32_baseline_close(oracle):
    z = np.load(GOLDEN / "small_matrix.npz")
    y = oracle.bf16_to_f32(oracle.qmm_f32(z["x"], z["w"], z["scales"], z["biases"]))
    rms = np.sqrt((z["y_r2"] ** 2).mean())
    assert np.abs(y - z["y_r2"]).max() <= 1e-2 * rms + 0.5 * np.abs(z["y_r2"]).max() * 2 ** -7


def test_qmm_f32_table_equals_exact_dequant(oracle):
    """The CPU baseline's fp32 R2 table reproduces the exact dequantized bits: with one-hot rows
    of x, y[m, n] = deq(W)[n, k_m] exactly."""
    kat = json.loads((GOLDEN / "deq_kat.json").read_text())["cases"]
    # keep every q of every group finite (0 * inf in an fp32 accumulation would be NaN)
    kat = [c for c in kat if (c["scale"] >> 7) & 0xFF < 240 and (c["bias"] >> 7) & 0xFF < 240][:512]
    N, G = 8, 64
    s = np.full((N, G), 0x3F80, dtype=np.uint16)
    b = np.zeros((N, G), dtype=np.uint16)
    for i, c in enumerate(kat):
        s[i // G, i % G], b[i // G, i % G] = c["scale"], c["bias"]
    w = np.random.default_rng(3).integers(0, 2 ** 32, size=(N, G * 8), dtype=np.uint32)
    K = G * 64
    ks = np.arange(0, K, 37)
    x = np.zeros((ks.size, K), dtype=np.uint16)
    x[np.arange(ks.size), ks] = 0x3F80
    y = oracle.qmm_f32(x, w, s, b)
    ref = oracle.dequantize(w, s, b)[:, ks].T
    zero = lambda a: np.where(a == 0x8000, 0, a)   # an fp32 sum starting at +0 turns -0 into +0
    assert (zero(y) == zero(ref)).all()


def test_layout_v1_fixture_and_roundtrip(oracle):
    z = np.load(GOLDEN / "small_matrix.npz")
    packed, sb = oracle.repack(z["w"], z["scales"], z["biases"])
    assert (packed == z["layout"]).all()
    assert (sb & 0xFFFF).reshape(2, 32).T.tolist() == z["scales"].tolist()
    w2, s2, b2 = oracle.unpack(packed, sb, 32, 128)
    assert (w2 == z["w"]).all() and (s2 == z["scales"]).all() and (b2 == z["biases"]).all()


def test_softcap_known_answers(oracle):
    kat = json.loads((GOLDEN / "softcap_kat.json").read_text())
    bad = [(h, e, oracle.softcap(h, kat["cap"])) for h, e in kat["cases"] if oracle.softcap(h, kat["cap"]) != e]
    assert not bad, bad[:5]


def test_tanh_accuracy(oracle):
    xs = np.linspace(-12, 12, 4001)
    err = max(abs(oracle.tanh(float(v)) - np.tanh(np.float64(np.float32(v)))) for v in xs)
    assert err < 2e-7


def test_argmax_first_index_wins_ties(oracle):
    logits = oracle.f32_to_bf16(np.array([1.0, 5.0, -3.0, 5.0, 4.99], dtype=np.float32))
    tok, val = oracle.softcap_argmax(logits, cap=0.0)
    assert tok == 1 and val == 5.0
    # softcap merges distinct logits into one bf16 value: the first of them wins
    big = oracle.f32_to_bf16(np.array([0.0, 120.0, 150.0, 3.0], dtype=np.float32))
    tok, val = oracle.softcap_argmax(big, cap=30.0)
    assert oracle.softcap(int(big[1])) == oracle.softcap(int(big[2]))
    assert tok == 1


def test_oracle_rejects_bad_format(oracle):
    z = np.load(GOLDEN / "small_matrix.npz")
    with pytest.raises(ValueError):
        oracle.dequantize(z["w"], z["scales"], z["biases"], group_size=48)
