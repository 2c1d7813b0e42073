"""Per-phase parity of one decode step of the synthetic stack against the CPU oracle (a checker).

Used by the GPU tests and, after its timed region, by bench.py's parity report. Every phase of
the step is checked on the GPU's own input for that phase ("teacher forced"): the oracle computes
the exact product of the bit-exact bf16 weights with the GPU's input rows, and the GPU's bf16
output must stay within the matmul contract max|y - y_oracle| <= 1e-2 * rms(y_oracle), beyond the
final bf16 rounding. The LM head is checked the same way on the GPU's final hidden state, and the
step's token must be exactly the first-index argmax of the softcapped GPU logits, and the oracle's
token up to a tie within one bf16 step of the softcapped value (0.125 near the cap).

The same oracle passes also carry the oracle's own chained step (the oracle's output fed to the
next phase, from the same h0) as second rows of each product, so the report gives the end-to-end
divergence too: after 193 bf16-rounded matmuls the GPU and oracle trajectories separate by rounding
flips alone, which is reported (rms-relative hidden difference, chained token) but is not the
per-phase contract.

The synthetic stack (matrix seeds, layer data flow) follows helios_b200/stack.py and the oracle's
stack_forward (oracle/affine.py); shapes are full width by default.
"""
from __future__ import annotations

import os

import numpy as np

from oracle import affine as A


def _half_ulp(v: np.ndarray) -> np.ndarray:
    a = np.abs(v).astype(np.float64)
    e = np.floor(np.log2(np.maximum(a, 2.0 ** -126)))
    return 0.5 * 2.0 ** (e - 7)


def _excess_ratio(y_bf16: np.ndarray, y_exact: np.ndarray) -> float:
    """max(|y - y_exact| - half an ulp of y_exact) / rms(y_exact)."""
    rms = float(np.sqrt(np.mean(y_exact.astype(np.float64) ** 2)))
    d = np.abs(A.bf16_to_f32(y_bf16).astype(np.float64) - y_exact) - _half_ulp(y_exact)
    return float(d.max()) / rms if rms > 0 else float(d.max())


def _rms_rows(x: np.ndarray, eps: float) -> np.ndarray:
    return np.array([A.rms_scale(x[m], eps) for m in range(x.shape[0])], dtype=np.float32)


def check_decode_step(shapes: dict, n_layers: int, h0: np.ndarray, layer_outs: list, token: list, value: list,
                      logits: np.ndarray | None = None, softcap: float = 30.0, eps: float = 1e-6) -> dict:
    """shapes: oracle stack_shapes(); h0: bf16 bits [M, hidden]; layer_outs[l]: dict of full-width
    bf16 bits qkv [M, q+2kv] (q|k|v), o [M, hidden], gu [M, 2*inter] (gate|up), h [M, hidden];
    token/value: the step's results per row; logits: the GPU's bf16 logits [M, vocab] or None."""
    M = h0.shape[0]
    A.set_threads(len(os.sched_getaffinity(0)))   # torchrun starts ranks with OMP_NUM_THREADS=1
    nq, nkv, ni = shapes["q"][0], shapes["k"][0], shapes["gate"][0]
    worst, worst_at = 0.0, ""
    per_kind = {"qkv": 0.0, "o": 0.0, "gu": 0.0, "down": 0.0}

    def record(kind, layer, ratio):
        nonlocal worst, worst_at
        per_kind[kind] = max(per_kind[kind], ratio)
        if ratio > worst:
            worst, worst_at = ratio, f"layer {layer} {kind}"

    x_g, x_c = np.ascontiguousarray(h0, dtype=np.uint16), np.ascontiguousarray(h0, dtype=np.uint16)
    for layer in range(n_layers):
        out = layer_outs[layer]
        X = np.vstack([x_g, x_c])
        r = _rms_rows(X, eps)
        chain_qkv = []
        col = 0
        for name in ("q", "k", "v"):
            n = shapes[name][0]
            ye, yb = A.qmm(X, *A.stack_matrix(layer, name, shapes), row_scale=r)
            record("qkv", layer, _excess_ratio(out["qkv"][:, col:col + n], ye[:M]))
            chain_qkv.append(yb[M:])
            col += n
        X = np.vstack([np.ascontiguousarray(out["qkv"][:, :nq]), chain_qkv[0]])
        ye, yb = A.qmm(X, *A.stack_matrix(layer, "o", shapes))
        record("o", layer, _excess_ratio(out["o"], ye[:M]))
        chain_o = yb[M:]
        X = np.vstack([np.ascontiguousarray(out["o"]), chain_o])
        r = _rms_rows(X, eps)
        chain_up = None
        for j, name in enumerate(("gate", "up")):
            ye, yb = A.qmm(X, *A.stack_matrix(layer, name, shapes), row_scale=r)
            record("gu", layer, _excess_ratio(out["gu"][:, j * ni:(j + 1) * ni], ye[:M]))
            chain_up = yb[M:]
        X = np.vstack([np.ascontiguousarray(out["gu"][:, ni:]), chain_up])
        ye, yb = A.qmm(X, *A.stack_matrix(layer, "down", shapes))
        record("down", layer, _excess_ratio(out["h"], ye[:M]))
        x_g, x_c = np.ascontiguousarray(out["h"]), yb[M:]
    X = np.vstack([x_g, x_c])
    ye, yb = A.qmm(X, *A.stack_matrix(0, "lm", shapes), row_scale=_rms_rows(X, eps))
    rep = {"phases": 4 * n_layers + 1, "max_excess_over_rms": round(worst, 6), "worst_phase": worst_at,
           "per_kind_max_excess_over_rms": {k: round(v, 6) for k, v in per_kind.items()}, "tolerance": 1e-2,
           "rows": M}
    tokens_ok = True
    tok_oracle, chain_tok = [], []
    for m in range(M):
        t_ref, v_ref = A.softcap_argmax(yb[m], softcap)          # the oracle's logits from the GPU's h
        tok_oracle.append(int(t_ref))
        tokens_ok &= int(token[m]) == int(t_ref) or abs(float(value[m]) - float(v_ref)) <= 0.125
        chain_tok.append(int(A.softcap_argmax(yb[M + m], softcap)[0]))
    if logits is not None:
        lm = _excess_ratio(logits, ye[:M])
        rep["lm_logits_excess_over_rms"] = round(lm, 6)
        rep["max_excess_over_rms"] = round(max(worst, lm), 6)
        if lm > worst:
            rep["worst_phase"] = "lm head"
        for m in range(M):    # the kernel's token is exactly the argmax of its own softcapped logits
            tokens_ok &= int(A.softcap_argmax(np.ascontiguousarray(logits[m]), softcap)[0]) == int(token[m])
    rep["token"] = [int(t) for t in token]
    rep["token_oracle"] = tok_oracle
    rep["token_match"] = bool(tokens_ok)
    hg = A.bf16_to_f32(x_g).astype(np.float64)
    hc = A.bf16_to_f32(x_c).astype(np.float64)
    rms_c = float(np.sqrt(np.mean(hc ** 2)))
    rep["chained"] = {"token": chain_tok, "hidden_rel_rms": round(float(np.sqrt(np.mean((hg - hc) ** 2))) / rms_c, 6),
                      "hidden_max_over_rms": round(float(np.abs(hg - hc).max()) / rms_c, 6)}
    rep["pass"] = bool(rep["max_excess_over_rms"] <= 1e-2 and tokens_ok)
    return rep
