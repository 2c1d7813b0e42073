"""GPU: the synthetic decoder stack end to end (fused q|k|v and gate|up launches, RMS scales
folded into epilogues, LM-head softcap + argmax) against the oracle's stack, eager and
replayed from a CUDA graph; plus error statuses of invalid calls (no GPU fault involved)."""
import numpy as np
import pytest
import torch

from gpu_util import qmm_error, u16

pytestmark = pytest.mark.gpu

SMALL = dict(layers=3, hidden=256, q_out=256, kv_out=128, inter=512, vocab=4096)


def oracle_stack(oracle, cfg, h0):
    shapes = oracle.stack_shapes(cfg.hidden, cfg.q_out, cfg.kv_out, cfg.inter, cfg.vocab)
    return oracle.stack_forward(h0, cfg.layers, shapes, cap=cfg.softcap, eps=cfg.eps)


@pytest.mark.parametrize("M", [1, 4])
def test_small_stack_matches_oracle(cuda, oracle, M):
    from helios_b200.quantized import synth_normal
    from helios_b200.stack import StackConfig, SyntheticStack, activation_seed, decode_keys
    cfg = StackConfig(**SMALL)
    st = SyntheticStack(cfg)
    h0 = synth_normal(activation_seed(M), (M, cfg.hidden))
    keys, h = st.forward(h0)
    ref = oracle_stack(oracle, cfg, u16(h0))
    excess, rms = qmm_error(oracle.bf16_to_f32(u16(h)), oracle.bf16_to_f32(ref["hidden"]).astype(np.float64),
                            bf16_out=True)
    assert excess <= 2e-2 * rms
    toks, vals = decode_keys(keys)
    for m in range(M):
        if toks[m] != ref["tokens"][m]:
            assert abs(vals[m] - ref["values"][m]) <= 0.125
    st.free()


def test_cuda_graph_replay_equals_eager(cuda, oracle):
    from helios_b200.quantized import synth_normal
    from helios_b200.stack import StackConfig, SyntheticStack, activation_seed
    cfg = StackConfig(**SMALL)
    st = SyntheticStack(cfg)
    static_h = synth_normal(activation_seed(0), (1, cfg.hidden))
    k_eager, h_eager = st.forward(static_h)
    k_eager, h_eager = k_eager.clone(), h_eager.clone()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        st.forward(static_h)     # warm-up on the capture stream
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        k_g, h_g = st.forward(static_h)
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(k_g, k_eager) and torch.equal(h_g, h_eager)
    static_h.copy_(synth_normal(activation_seed(5), (1, cfg.hidden)))
    g.replay()
    k2, h2 = st.forward(static_h.clone())
    torch.cuda.synchronize()
    assert torch.equal(k_g, k2)
    del g
    st.free()


PLAN = dict(layers=2, hidden=2048, q_out=2048, kv_out=1024, inter=4096, vocab=16384)


def test_decode_plan_single_launch(cuda, oracle):
    """The persistent decode-step kernel (one launch for all phases) against the per-matmul path
    and the oracle; bit-reproducible across runs and under CUDA-graph replay."""
    from helios_b200 import _lib
    from helios_b200.quantized import synth_normal
    from helios_b200.stack import StackConfig, SyntheticStack, activation_seed, decode_keys
    cfg = StackConfig(**PLAN)
    st = SyntheticStack(cfg)
    h0 = synth_normal(activation_seed(3), (1, cfg.hidden))
    k_eager, h_eager = st.forward(h0)
    k_eager, h_eager = k_eager.clone(), h_eager.clone()
    st.build_plan(1)
    k1, h1 = st.decode(h0)
    k1, h1 = k1.clone(), h1.clone()
    assert _lib.device_error() == 0
    ex, rms = qmm_error(oracle.bf16_to_f32(u16(h1)), oracle.bf16_to_f32(u16(h_eager)).astype(np.float64), True)
    assert ex <= 2e-2 * rms
    k2, h2 = st.decode(h0)
    assert torch.equal(k2, k1) and torch.equal(h2, h1)          # deterministic reductions
    ref = oracle_stack(oracle, cfg, u16(h0))
    t1, v1 = decode_keys(k1)
    assert t1[0] == ref["tokens"][0] or abs(v1[0] - ref["values"][0]) <= 0.125
    # graph replay of the single launch
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        st.decode(h0)
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        kg, hg = st.decode(h0)
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    assert torch.equal(kg, k1) and torch.equal(hg, h1)
    assert _lib.device_error() == 0
    del g
    st.free()


def test_decode_plan_regular_last_phase(cuda, oracle):
    """A plan that ends with a plain matmul (no argmax): y1 = rms(x) * x W1^T, y2 = y1 W2^T. The last
    phase's cut quads are written back after every CTA has finished it."""
    from helios_b200 import _lib
    from helios_b200 import quantized as Q
    N1, K1, N2 = 2048, 2048, 1536
    mats = [oracle.synth_matrix(oracle.matrix_seed(5, i), n, k) for i, (n, k) in enumerate(((N1, K1), (N2, N1)))]
    ws = [Q.QuantizedWeight.from_mlx(torch.from_numpy(w.view(np.int32)).view(torch.uint32),
                                     torch.from_numpy(s.view(np.int16)).view(torch.bfloat16),
                                     torch.from_numpy(b.view(np.int16)).view(torch.bfloat16)) for w, s, b in mats]
    x = Q.synth_normal(oracle.activation_seed(41), (1, K1))
    y1 = torch.empty((1, N1), dtype=torch.bfloat16, device=cuda)
    y2 = torch.empty((1, N2), dtype=torch.bfloat16, device=cuda)
    plan = Q.DecodePlan([(ws[0], x, y1, Q.QMM_RMS_SCALE), (ws[1], y1, y2, 0)], 1)
    for _ in range(2):
        y2.fill_(float("nan"))
        plan.run(1)
        torch.cuda.synchronize()
        assert _lib.device_error() == 0
        r = np.array([oracle.rms_scale(u16(x)[0], 1e-6)], dtype=np.float32)
        ref1 = oracle.qmm(u16(x), *mats[0], row_scale=r)[0]
        ex, rms = qmm_error(oracle.bf16_to_f32(u16(y1)), ref1, True)
        assert ex <= 1e-2 * rms
        ref2 = oracle.qmm(u16(y1), *mats[1])[0]     # the second phase from the first phase's own output
        ex, rms = qmm_error(oracle.bf16_to_f32(u16(y2)), ref2, True)
        assert ex <= 1e-2 * rms
    plan.free()
    for w in ws:
        w.free()


def test_decode_plan_rejects_bad_phases(cuda, oracle):
    from helios_b200 import _lib
    from helios_b200 import quantized as Q
    w = Q.QuantizedWeight.from_mlx(*Q.synth_matrix(1, 64, 256))
    x = torch.zeros((1, 256), dtype=torch.bfloat16, device=cuda)
    y = torch.zeros((1, 64), dtype=torch.bfloat16, device=cuda)
    with pytest.raises(_lib.G4qError):                       # too few units for a full grid
        Q.DecodePlan([(w, x, y, 0)])
    big = Q.QuantizedWeight.from_mlx(*Q.synth_matrix(2, 4096, 4096))
    xb = torch.zeros((1, 4096), dtype=torch.bfloat16, device=cuda)
    yb = torch.zeros((1, 4096), dtype=torch.bfloat16, device=cuda)
    with pytest.raises(_lib.G4qInvalidArgument):              # argmax phase must be last
        Q.DecodePlan([(big, xb, yb, Q.PHASE_ARGMAX), (big, yb, xb, 0)])
    for m in (3, 16):                                         # token counts the plan does not take
        with pytest.raises(_lib.G4qError):
            Q.DecodePlan([(big, xb, yb, 0)], max_tokens=m)
    w.free()
    big.free()


def test_invalid_calls_return_status(cuda, oracle):
    from helios_b200 import _lib
    from helios_b200 import quantized as Q
    w, s, b = Q.synth_matrix(1, 64, 256)
    with pytest.raises(_lib.G4qError) as e:
        Q.QuantizedWeight(60, 256)                       # rows % 16 != 0
    assert e.value.status == _lib.G4Q_ERR_UNSUPPORTED_CONFIG
    for bits, gs in ((2, 64), (3, 64), (4, 48), (8, 256)):   # specs the manifest never names
        with pytest.raises(_lib.G4qError) as e:
            Q.QuantizedWeight(64, 256, bits=bits, group_size=gs)
        assert e.value.status == _lib.G4Q_ERR_UNSUPPORTED_CONFIG
    q = Q.QuantizedWeight.from_mlx(w, s, b)
    with pytest.raises(ValueError):
        Q.quantized_matmul(torch.zeros((1, 128), dtype=torch.bfloat16, device=cuda), q)   # K mismatch
    with pytest.raises(_lib.G4qInvalidArgument):
        q.load(w, s, b, src_row=32, n_rows=48)           # window past the source
    with pytest.raises(_lib.G4qInvalidArgument):
        _lib.call("g4q_qmm", q.handle, 12345, 1, 256, 0, 64, None)   # misaligned x (checked on host)
    with pytest.raises(_lib.G4qInvalidArgument):
        Q.lm_head_argmax(torch.zeros((17, 256), dtype=torch.bfloat16, device=cuda), q)   # M > 16
    # a huge scale disables the fast path with a clear status, while dequantize still works
    s2 = s.clone()
    s2[0, 0] = torch.tensor(2.0 ** 121, dtype=torch.bfloat16)
    q2 = Q.QuantizedWeight.from_mlx(w, s2, b)
    assert q2.info()["fast_path_ok"] == 0
    with pytest.raises(_lib.G4qError) as e:
        Q.quantized_matmul(torch.zeros((1, 256), dtype=torch.bfloat16, device=cuda), q2)
    assert e.value.status == _lib.G4Q_ERR_UNSUPPORTED_CONFIG
    Q.dequantize(q2)
    torch.cuda.synchronize()
    q.free()
    q2.free()
    with pytest.raises(ValueError):
        q.handle
