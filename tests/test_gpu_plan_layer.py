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


def _excess(y_bits, y_exact):
    from stack_parity import _excess_ratio
    return _excess_ratio(y_bits, y_exact)


def _close_residual(A, got, want, tag):
    g, w = A.bf16_to_f32(got).astype(np.float64), A.bf16_to_f32(want).astype(np.float64)
    rms = float(np.sqrt(np.mean(w ** 2)))
    bad = np.count_nonzero(got != want)
    assert bad <= max(2, got.size // 1000), f"{tag}: {bad} of {got.size} residual values differ"
    assert float(np.abs(g - w).max()) <= 1e-2 * rms, f"{tag}: residual differs by more than 1e-2 * rms"


@pytest.fixture(scope="module")
def layers(cuda):
    """helios_b200.stack.DecoderStack: the real layer structure, seeded synthetic weights."""
    from helios_b200.stack import DecoderStack, StackConfig
    st = DecoderStack(StackConfig(layers=LAYERS), max_tokens=8)
    yield st
    st.free()


@pytest.mark.parametrize("M", [1, 2, 8])
def test_real_layer_plan_every_phase(cuda, oracle, layers, M):
    from helios_b200 import _lib
    from helios_b200.quantized import synth_normal
    from helios_b200.stack import activation_seed
    A, c = oracle, layers.cfg
    A.set_threads(len(os.sched_getaffinity(0)))
    shapes = A.stack_shapes()
    layers.build_plan(M, keep_layers=True)
    h0 = synth_normal(activation_seed(100 + M), (M, c.hidden))
    logits = torch.empty((M, c.vocab), dtype=torch.bfloat16, device=cuda)
    layers.decode(h0, logits=logits)
    torch.cuda.synchronize()
    tokens, values = layers.tokens[:M], layers.values[:M]
    assert _lib.device_error() == 0
    nw = {k: u16(v) for k, v in (("final", layers.final_norm),)}
    res_prev = None
    worst = {}
    for i, L in enumerate(layers.layers):
        b = {k: u16(v) for k, v in layers.outs[i].items()}
        w = {k: u16(L[k]) for k in ("in_norm", "post_attn", "pre_ffn", "post_ffn")}
        # the residual stream before the layer and the normalized input of qkv
        if i == 0:
            assert np.array_equal(b["res_a"], u16(h0)), "the first phase starts the residual stream with x"
        else:
            P = layers.layers[i - 1]
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
    P = layers.layers[-1]
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
    layers.decode(h0, logits=logits)
    torch.cuda.synchronize()
    again = [u16(t) for b in layers.outs for t in b.values()] + [u16(logits), u16(layers.res_final)]
    assert all(np.array_equal(x, y) for x, y in zip(first, again))


def test_prologue_validation(cuda, layers):
    """Prologue rules the plan enforces before anything runs."""
    from helios_b200.quantized import QMM_RMS_SCALE, PHASE_ARGMAX, DecodePlan, G4qError
    c, L = layers.cfg, layers.layers[0]
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
