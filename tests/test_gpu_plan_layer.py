"""GPU: decode plans of real decoder layers -- the norms, residual stream, layer scalar and GeGLU
inside the persistent decode kernel -- every phase against the oracle on its own GPU input.

Per layer (native_model.cc:899-970 layer_forward, with attention left out: q stands in for the
attention output, as in the synthetic stack):

    phase qkv   prologue: [post_feedforward_layernorm of the previous layer, residual add,
                layer_scalar] then input_layernorm; x = the previous layer's down output
                (layer 0: the step's input h, which starts the residual stream)
    phase o     x = q (a column window of the qkv output)
    phase gu    prologue: post_attention_layernorm, residual add, pre_feedforward_layernorm;
                paired gate|up weight with the GeGLU in the epilogue
    phase down  x = the GeGLU output
    LM head     prologue: the last layer's post-feedforward norm, residual add and scalar, then
                the final norm; argmax of the softcapped logits

Every residual-stream value the plan produces (its ``residual_out`` copies) must equal the oracle's
norm + residual + scalar of the GPU's own inputs except for rare one-ulp flips of the normalized
value (the fp32 sum of squares is accumulated in another order than the oracle's float64 mean);
every matmul output must meet the matmul contract (max excess <= 1e-2 * rms) against the exact
product of the oracle's normalized input; the GeGLU output must equal the oracle's GeGLU of the
exact gate/up products rounded to bf16 except where a gate/up rounding flipped (at most 1 % of the
values, each within 1e-2 * rms + 2^-6 * |value|).
"""
import os

import numpy as np
import pytest
import torch

from gpu_util import u16

pytestmark = pytest.mark.gpu

LAYERS = 2


def _norm_weight(seed, n, device):
    from helios_b200.quantized import synth_normal
    return (synth_normal(seed, (n,)).float() * 0.1 + 1.0).to(torch.bfloat16).to(device)


def _excess(y_bits, y_exact):
    from stack_parity import _excess_ratio
    return _excess_ratio(y_bits, y_exact)


def _close_residual(A, got, want, tag):
    g, w = A.bf16_to_f32(got).astype(np.float64), A.bf16_to_f32(want).astype(np.float64)
    rms = float(np.sqrt(np.mean(w ** 2)))
    bad = np.count_nonzero(got != want)
    assert bad <= max(2, got.size // 1000), f"{tag}: {bad} of {got.size} residual values differ"
    assert float(np.abs(g - w).max()) <= 1e-2 * rms, f"{tag}: residual differs by more than 1e-2 * rms"


class _Layers:
    """Real-layer weights on the GPU (paired gate|up) and their norm weights and scalars."""

    def __init__(self, device, cfg):
        from helios_b200.quantized import QuantizedWeight, synth_matrix
        from helios_b200.stack import matrix_seed
        sh = cfg.shapes()
        self.cfg, self.L = cfg, []
        for layer in range(LAYERS):
            mats = {p: synth_matrix(matrix_seed(layer, p), *sh[p]) for p in ("q", "k", "v")}
            qkv = QuantizedWeight.concat([mats["q"], mats["k"], mats["v"]])
            del mats
            o = QuantizedWeight.from_mlx(*synth_matrix(matrix_seed(layer, "o"), *sh["o"]))
            gu = QuantizedWeight.geglu_pair(synth_matrix(matrix_seed(layer, "gate"), *sh["gate"]),
                                            synth_matrix(matrix_seed(layer, "up"), *sh["up"]))
            down = QuantizedWeight.from_mlx(*synth_matrix(matrix_seed(layer, "down"), *sh["down"]))
            s = 1000 + 10 * layer
            self.L.append({"qkv": qkv, "o": o, "gu": gu, "down": down,
                           "in_norm": _norm_weight(s, cfg.hidden, device),
                           "post_attn": _norm_weight(s + 1, cfg.hidden, device),
                           "pre_ffn": _norm_weight(s + 2, cfg.hidden, device),
                           "post_ffn": _norm_weight(s + 3, cfg.hidden, device),
                           "scalar": torch.tensor([0.75 - 0.125 * layer], dtype=torch.bfloat16, device=device)})
        self.lm = QuantizedWeight.from_mlx(*synth_matrix(matrix_seed(0, "lm"), *sh["lm"]))
        self.final_norm = _norm_weight(999, cfg.hidden, device)

    def plan(self, M, device):
        from helios_b200.quantized import PHASE_ARGMAX, PHASE_GEGLU, DecodePlan
        c = self.cfg
        bf = dict(dtype=torch.bfloat16, device=device)
        self.h_in = torch.zeros((M, c.hidden), **bf)
        self.outs = []
        phases, pro, x = [], [], self.h_in
        for i, L in enumerate(self.L):
            b = {"qkv": torch.empty((M, c.q_out + 2 * c.kv_out), **bf), "o": torch.empty((M, c.hidden), **bf),
                 "act": torch.empty((M, c.inter), **bf), "h": torch.empty((M, c.hidden), **bf),
                 "res_a": torch.empty((M, c.hidden), **bf), "res_b": torch.empty((M, c.hidden), **bf)}
            self.outs.append(b)
            if i == 0:
                pro.append({"residual": 1, "norm_weight": L["in_norm"], "residual_out": b["res_a"], "eps": c.eps})
            else:
                P = self.L[i - 1]
                pro.append({"post_norm_weight": P["post_ffn"], "residual": 2, "layer_scalar": P["scalar"],
                            "norm_weight": L["in_norm"], "residual_out": b["res_a"], "eps": c.eps})
            phases.append((L["qkv"], x, b["qkv"], 0))
            pro.append(None)
            phases.append((L["o"], b["qkv"][:, : c.q_out], b["o"], 0))
            pro.append({"post_norm_weight": L["post_attn"], "residual": 2, "norm_weight": L["pre_ffn"],
                        "residual_out": b["res_b"], "eps": c.eps})
            phases.append((L["gu"], b["o"], b["act"], PHASE_GEGLU))
            pro.append(None)
            phases.append((L["down"], b["act"], b["h"], 0))
            x = b["h"]
        P = self.L[-1]
        self.res_final = torch.empty((M, c.hidden), **bf)
        pro.append({"post_norm_weight": P["post_ffn"], "residual": 2, "layer_scalar": P["scalar"],
                    "norm_weight": self.final_norm, "residual_out": self.res_final, "eps": c.eps})
        phases.append((self.lm, x, None, PHASE_ARGMAX))
        return DecodePlan(phases, M, prologues=pro)


@pytest.fixture(scope="module")
def layers(cuda):
    from helios_b200.stack import StackConfig
    return _Layers(cuda, StackConfig(layers=LAYERS))


@pytest.mark.parametrize("M", [1, 2])
def test_real_layer_plan_every_phase(cuda, oracle, layers, M):
    from helios_b200 import _lib
    from helios_b200.quantized import synth_normal
    from helios_b200.stack import activation_seed, decode_keys
    A, c = oracle, layers.cfg
    A.set_threads(len(os.sched_getaffinity(0)))
    shapes = A.stack_shapes()
    plan = layers.plan(M, cuda)
    h0 = synth_normal(activation_seed(100 + M), (M, c.hidden))
    layers.h_in.copy_(h0)
    logits = torch.empty((M, c.vocab), dtype=torch.bfloat16, device=cuda)
    tokens = torch.empty(M, dtype=torch.int32, device=cuda)
    values = torch.empty(M, dtype=torch.float32, device=cuda)
    keys = torch.empty(M, dtype=torch.int64, device=cuda)
    plan.run(M, softcap=c.softcap, tokens=tokens, values=values, keys=keys, logits=logits)
    torch.cuda.synchronize()
    assert _lib.device_error() == 0
    nw = {k: u16(v) for k, v in (("final", layers.final_norm),)}
    res_prev = None
    worst = {}
    for i, L in enumerate(layers.L):
        b = {k: u16(v) for k, v in layers.outs[i].items()}
        w = {k: u16(L[k]) for k in ("in_norm", "post_attn", "pre_ffn", "post_ffn")}
        # the residual stream before the layer and the normalized input of qkv
        if i == 0:
            assert np.array_equal(b["res_a"], u16(h0)), "the first phase starts the residual stream with x"
        else:
            P = layers.L[i - 1]
            want = A.rms_norm_residual(u16(layers.outs[i - 1]["h"]), u16(P["post_ffn"]), res_prev,
                                       int(u16(P["scalar"])[0]), c.eps)
            _close_residual(A, b["res_a"], want, f"layer {i} input residual")
        xn = A.rms_norm(b["res_a"], w["in_norm"], c.eps)
        col = 0
        for name in ("q", "k", "v"):
            n = shapes[name][0]
            ye, _ = A.qmm(xn, *A.stack_matrix(i, name, shapes))
            worst[f"{i} {name}"] = _excess(b["qkv"][:, col:col + n], ye)
            col += n
        ye, _ = A.qmm(np.ascontiguousarray(b["qkv"][:, : c.q_out]), *A.stack_matrix(i, "o", shapes))
        worst[f"{i} o"] = _excess(b["o"], ye)
        want = A.rms_norm_residual(b["o"], w["post_attn"], b["res_a"], None, c.eps)
        _close_residual(A, b["res_b"], want, f"layer {i} attention residual")
        xn = A.rms_norm(b["res_b"], w["pre_ffn"], c.eps)
        g_e, g_b = A.qmm(xn, *A.stack_matrix(i, "gate", shapes))
        u_e, u_b = A.qmm(xn, *A.stack_matrix(i, "up", shapes))
        act = A.geglu(g_b, u_b)
        af, gf = A.bf16_to_f32(act).astype(np.float64), A.bf16_to_f32(b["act"]).astype(np.float64)
        rms = float(np.sqrt(np.mean(af ** 2)))
        diff = np.count_nonzero(b["act"] != act)
        assert diff <= act.size // 100, f"layer {i}: {diff} of {act.size} GeGLU values differ"
        assert np.all(np.abs(gf - af) <= 1e-2 * rms + 2.0 ** -6 * np.abs(af)), f"layer {i}: GeGLU values"
        ye, _ = A.qmm(b["act"], *A.stack_matrix(i, "down", shapes))
        worst[f"{i} down"] = _excess(b["h"], ye)
        res_prev = b["res_b"]
    P = layers.L[-1]
    want = A.rms_norm_residual(u16(layers.outs[-1]["h"]), u16(P["post_ffn"]), res_prev, int(u16(P["scalar"])[0]),
                               c.eps)
    rf = u16(layers.res_final)
    _close_residual(A, rf, want, "final residual")
    xn = A.rms_norm(rf, nw["final"], c.eps)
    ye, yb = A.qmm(xn, *A.stack_matrix(0, "lm", shapes))
    lg = u16(logits)
    worst["lm"] = _excess(lg, ye)
    assert max(worst.values()) <= 1e-2, worst
    tk = tokens.cpu().numpy()
    for m in range(M):
        t_own, _ = A.softcap_argmax(np.ascontiguousarray(lg[m]), c.softcap)
        assert int(tk[m]) == int(t_own)
        t_ref, v_ref = A.softcap_argmax(np.ascontiguousarray(yb[m]), c.softcap)
        assert int(tk[m]) == int(t_ref) or abs(float(values[m]) - float(v_ref)) <= 0.125
    # a second step from the same input reproduces every output bit for bit
    first = [u16(t) for b in layers.outs for t in b.values()] + [lg, rf]
    plan.run(M, softcap=c.softcap, tokens=tokens, values=values, keys=keys, logits=logits)
    torch.cuda.synchronize()
    again = [u16(t) for b in layers.outs for t in b.values()] + [u16(logits), u16(layers.res_final)]
    assert all(np.array_equal(x, y) for x, y in zip(first, again))
    plan.free()


def test_prologue_validation(cuda, layers):
    """Prologue rules the plan enforces before anything runs."""
    from helios_b200.quantized import QMM_RMS_SCALE, PHASE_ARGMAX, DecodePlan, G4qError
    c, L = layers.cfg, layers.L[0]
    bf = dict(dtype=torch.bfloat16, device=cuda)
    x = torch.zeros((1, c.hidden), **bf)
    qkv = torch.empty((1, c.q_out + 2 * c.kv_out), **bf)
    o = torch.empty((1, c.hidden), **bf)
    base = [(L["qkv"], x, qkv, 0), (L["o"], qkv[:, : c.q_out], o, 0), (layers.lm, o, None, PHASE_ARGMAX)]
    bad = [
        # a residual add with no residual stream started before it
        [{"residual": 2, "norm_weight": L["in_norm"]}, None, None],
        # a layer scalar without a residual add
        [{"residual": 1, "layer_scalar": L["scalar"]}, None, None],
        # a prologue on a phase that reads a column window of the previous output
        [{"residual": 1}, {"norm_weight": L["in_norm"]}, None],
    ]
    for pro in bad:
        with pytest.raises(G4qError):
            DecodePlan(base, 1, prologues=pro)
    rms = [(L["qkv"], x, qkv, QMM_RMS_SCALE)] + base[1:]
    with pytest.raises(G4qError):   # a prologue phase takes no RMS scale of its own
        DecodePlan(rms, 1, prologues=[{"norm_weight": L["in_norm"]}, None, None])
    with pytest.raises(ValueError):
        DecodePlan(base, 1, prologues=[None])
    DecodePlan(base, 1, prologues=[{"residual": 1, "norm_weight": L["in_norm"]}, None,
                                   {"post_norm_weight": L["post_attn"], "residual": 2,
                                    "norm_weight": layers.final_norm}]).free()
