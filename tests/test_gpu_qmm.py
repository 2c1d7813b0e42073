"""GPU: quantized matmul (decode GEMV M <= 16, prefill GEMM M > 16) and the fused LM-head
softcap + argmax against the CPU oracle, through the C ABI.

Tolerance (north star): max|y - y_oracle| <= 1e-2 * rms(y_oracle), with y_oracle the exact
(float64) product of the bit-exact bf16 dequantized weights. For bf16 outputs the final
bf16 rounding (half an ulp of the value) is excluded: the oracle's own bf16 output exceeds
the raw bound by up to 1.7e-2 * rms on outliers beyond 16 at these shapes. fp32 outputs are
checked against the raw bound."""
import numpy as np
import pytest
import torch

from gpu_util import assert_qmm_close, dev_u16, qmm_error, u16

pytestmark = pytest.mark.gpu

SHAPES = {"q": (4096, 3840), "k": (2048, 3840), "o": (3840, 4096), "gate": (15360, 3840), "down": (3840, 15360)}


def make(oracle, Q, proj, N, K, M, layer=0, chunk=0):
    seed = oracle.matrix_seed(layer, oracle.PROJ_IDS[proj])
    w, s, b = Q.synth_matrix(seed, N, K)
    qw = Q.QuantizedWeight.from_mlx(w, s, b)
    x = Q.synth_normal(oracle.activation_seed(chunk), (M, K))
    ow, os_, ob = oracle.synth_matrix(seed, N, K)
    return qw, x, (ow, os_, ob)


@pytest.mark.parametrize("proj", list(SHAPES))
@pytest.mark.parametrize("M", [1, 2, 4, 8])
def test_decode_gemv_baseline_shapes(cuda, oracle, proj, M):
    from helios_b200 import quantized as Q
    N, K = SHAPES[proj]
    qw, x, (ow, os_, ob) = make(oracle, Q, proj, N, K, M, chunk=M)
    # every BASELINE shape at M <= 8 runs the stream-K GEMV (down_proj at M = 8 with 12 warps per CTA)
    from helios_b200 import _lib
    assert qw.qmm_path(M) == (_lib.PATH_GEMV_STREAMK, 0)
    ye, yb = oracle.qmm(u16(x), ow, os_, ob)
    y = Q.quantized_matmul(x, qw)
    assert y.shape == (M, N) and y.dtype == torch.bfloat16
    yg = oracle.bf16_to_f32(u16(y))
    assert_qmm_close(yg, ye, bf16_out=True)
    assert (u16(y) == yb).mean() > 0.99       # bit-equal bf16 except rare 1-ulp rounding flips
    yf = Q.quantized_matmul(x, qw, out_dtype=torch.float32).cpu().numpy()
    assert_qmm_close(yf, ye, bf16_out=False)
    qw.free()


@pytest.mark.parametrize("M", [3, 5, 9, 15, 16])
def test_decode_gemv_odd_widths(cuda, oracle, M):
    from helios_b200 import quantized as Q
    qw, x, (ow, os_, ob) = make(oracle, Q, "q", 4096, 3840, M, layer=3, chunk=100 + M)
    ye, _ = oracle.qmm(u16(x), ow, os_, ob)
    yf = Q.quantized_matmul(x, qw, out_dtype=torch.float32).cpu().numpy()
    assert_qmm_close(yf, ye, bf16_out=False)
    qw.free()


FULL_ATTENTION = {"q_full": (8192, 3840), "k_full": (512, 3840), "o_full": (3840, 8192)}


@pytest.mark.parametrize("proj", list(FULL_ATTENTION))
@pytest.mark.parametrize("M", [1, 8, 15, 64])
def test_full_attention_layer_shapes(cuda, oracle, proj, M):
    """The real model's every-sixth layer (native_model.cc:496-498, 788-897): head_dim 512 and one
    KV head, so q 8192x3840, k 512x3840 (no v) and o 3840x8192; at decode (1), MTP verify (8, 15:
    decode_block_logits, :2006) and a prefill width (64)."""
    from helios_b200 import quantized as Q
    N, K = FULL_ATTENTION[proj]
    qw, x, (ow, os_, ob) = make(oracle, Q, "q" if proj != "o_full" else "o", N, K, M, layer=5, chunk=200 + M)
    ye, yb = oracle.qmm(u16(x), ow, os_, ob)
    y = Q.quantized_matmul(x, qw)
    assert_qmm_close(oracle.bf16_to_f32(u16(y)), ye, bf16_out=True)
    assert (u16(y) == yb).mean() > 0.99
    qw.free()


# The 12B MTP assistant (config checked at native/gemma4_mlx/src/model_manifest.cc:265-272: hidden
# 1024, intermediate 8192, 16 heads of 256, head_dim 512 on its full-attention layer 3, no k/v
# projections) and its linears (native_model.cc:2134-2243): pre_projection over the concatenated
# token embedding and target hidden (3840 + 3840 -> 1024), post_projection back to 3840.
ASSISTANT = {"pre_projection": (1024, 7680), "q": (4096, 1024), "q_full": (8192, 1024), "o": (1024, 4096),
             "o_full": (1024, 8192), "gate_up": (8192, 1024), "down": (1024, 8192), "post_projection": (3840, 1024)}


@pytest.mark.parametrize("name", list(ASSISTANT))
@pytest.mark.parametrize("M", [1, 4])
def test_mtp_assistant_shapes(cuda, oracle, name, M):
    from helios_b200 import quantized as Q
    N, K = ASSISTANT[name]
    qw, x, (ow, os_, ob) = make(oracle, Q, "up", N, K, M, layer=40, chunk=300 + M)
    ye, yb = oracle.qmm(u16(x), ow, os_, ob)
    y = Q.quantized_matmul(x, qw)
    assert_qmm_close(oracle.bf16_to_f32(u16(y)), ye, bf16_out=True)
    assert (u16(y) == yb).mean() > 0.99
    qw.free()


def test_mtp_assistant_lm_head_without_softcap(cuda, oracle):
    """assistant_logits (native_model.cc:2103-2116): the assistant's tied 262144 x 1024 head, bf16
    logits with no softcap, then a greedy argmax (:2227)."""
    from helios_b200 import quantized as Q
    N, K = 262144, 1024
    seed = oracle.matrix_seed(41, 7)
    w, s, b = Q.synth_matrix(seed, N, K)
    qw = Q.QuantizedWeight.from_mlx(w, s, b)
    x = Q.synth_normal(oracle.activation_seed(41), (1, K))
    logits = torch.empty((1, N), dtype=torch.bfloat16, device=cuda)
    tok, val, _ = Q.lm_head_argmax(x, qw, softcap=0.0, logits=logits)
    ow, os_, ob = oracle.synth_matrix(seed, N, K)
    ye, yb = oracle.qmm(u16(x), ow, os_, ob)
    assert_qmm_close(oracle.bf16_to_f32(u16(logits)), ye, bf16_out=True)
    t_self, v_self = oracle.softcap_argmax(u16(logits[0]), 0.0)
    assert int(tok[0]) == t_self and float(val[0]) == v_self
    t_ref, v_ref = oracle.softcap_argmax(yb[0], 0.0)
    assert int(tok[0]) == t_ref or abs(v_self - v_ref) <= 0.125
    qw.free()


@pytest.mark.parametrize("N,K", [(16, 64), (48, 192), (80, 1024), (272, 640), (128, 768), (320, 192),
                                 (1088, 512)])
@pytest.mark.parametrize("M", [1, 7, 16])
def test_ragged_small_shapes(cuda, oracle, N, K, M):
    """Small and ragged shapes: N not a multiple of 64 (cluster split-K kernel), and tiny stream-K
    grids where one 64-row quad is reduced from many warps' partial sums."""
    from helios_b200 import quantized as Q
    w, s, b = oracle.synth_matrix(N * 7 + K, N, K)
    x = oracle.synth_normal_bf16(N + K + M, M * K).reshape(M, K)
    qw = Q.QuantizedWeight.from_mlx(torch.from_numpy(w.view(np.int32)).view(torch.uint32),
                                    torch.from_numpy(s.view(np.int16)).view(torch.bfloat16),
                                    torch.from_numpy(b.view(np.int16)).view(torch.bfloat16))
    ye, _ = oracle.qmm(x, w, s, b)
    yf = Q.quantized_matmul(dev_u16(x, cuda), qw, out_dtype=torch.float32).cpu().numpy()
    assert_qmm_close(yf, ye, bf16_out=False)
    qw.free()


def test_stream_k_is_deterministic(cuda, oracle):
    """Split quads are summed in a fixed contributor order: repeated launches are bit-identical."""
    from helios_b200 import _lib
    from helios_b200 import quantized as Q
    qw, x, _ = make(oracle, Q, "down", 3840, 15360, 1, layer=2)
    ys = [Q.quantized_matmul(x, qw, out_dtype=torch.float32) for _ in range(3)]
    assert all(torch.equal(ys[0], y) for y in ys[1:])
    assert _lib.device_error() == 0
    qw.free()


def test_rms_scale_and_strided_input(cuda, oracle):
    """RMS_SCALE folds 1/sqrt(mean(x^2)+eps) into the output; x may be a strided column slice."""
    from helios_b200 import quantized as Q
    qw, _, (ow, os_, ob) = make(oracle, Q, "o", 3840, 4096, 1)
    big = Q.synth_normal(oracle.activation_seed(9), (4, 8192)) * 3.0
    x = big[:, 1024:1024 + 4096]                     # row stride 8192, 16-byte aligned
    xn = u16(x.contiguous())
    r = np.array([oracle.rms_scale(xn[m]) for m in range(4)], dtype=np.float32)
    ye, _ = oracle.qmm(xn, ow, os_, ob, row_scale=r)
    yf = Q.quantized_matmul(x, qw, rms_scale=True, out_dtype=torch.float32).cpu().numpy()
    assert_qmm_close(yf, ye, bf16_out=False)
    qw.free()


@pytest.mark.parametrize("M", [17, 64, 200])
def test_prefill_widths_small_n(cuda, oracle, M):
    from helios_b200 import quantized as Q
    qw, x, (ow, os_, ob) = make(oracle, Q, "k", 2048, 3840, M, layer=5, chunk=M)
    ye, _ = oracle.qmm(u16(x), ow, os_, ob)
    yf = Q.quantized_matmul(x, qw, out_dtype=torch.float32).cpu().numpy()
    assert_qmm_close(yf, ye, bf16_out=False)
    qw.free()


@pytest.mark.parametrize("M,N,K", [(100, 1920, 3840), (129, 272, 640), (300, 3840, 4096)])
def test_prefill_gemm_ragged_rms_f32(cuda, oracle, M, N, K):
    """tcgen05 GEMM: M not a multiple of 128, N not a multiple of 256 (TP-8 gate shard, 17 row
    tiles), RMS row scale and fp32 output; no bounded wait may have given up."""
    from helios_b200 import _lib
    from helios_b200 import quantized as Q
    seed = oracle.matrix_seed(2, 4) ^ N
    w, s, b = Q.synth_matrix(seed, N, K)
    qw = Q.QuantizedWeight.from_mlx(w, s, b)
    x = Q.synth_normal(oracle.activation_seed(M), (M, K))
    xn = u16(x)
    ow, os_, ob = oracle.synth_matrix(seed, N, K)
    r = np.array([oracle.rms_scale(xn[m]) for m in range(M)], dtype=np.float32)
    ye, _ = oracle.qmm(xn, ow, os_, ob, row_scale=r)
    yf = Q.quantized_matmul(x, qw, rms_scale=True, out_dtype=torch.float32).cpu().numpy()
    assert_qmm_close(yf, ye, bf16_out=False)
    yb = Q.quantized_matmul(x, qw, rms_scale=True)
    assert_qmm_close(oracle.bf16_to_f32(u16(yb)), ye, bf16_out=True)
    assert _lib.device_error() == 0
    qw.free()


def test_prefill_chunk_2048(cuda, oracle):
    """A full 2048-token prefill chunk (BASELINE config 3 width) on a 256-row slice of up_proj."""
    from helios_b200 import quantized as Q
    seed = oracle.matrix_seed(0, 5)
    w, s, b = Q.synth_matrix(seed, 15360, 3840)
    qw = Q.QuantizedWeight.from_mlx(w, s, b, rows=(4096, 4352))
    x = Q.synth_normal(oracle.activation_seed(1), (2048, 3840))
    ow, os_, ob = oracle.synth_matrix(seed, 15360, 3840)
    ye, _ = oracle.qmm(u16(x), ow[4096:4352], os_[4096:4352], ob[4096:4352])
    yb = Q.quantized_matmul(x, qw)
    assert_qmm_close(oracle.bf16_to_f32(u16(yb)), ye, bf16_out=True)
    qw.free()


def test_prefill_gemm_unsplit_up_slice_2048(cuda, oracle):
    """The GEMM path the prefill benchmark times: 2048 tokens on 2560 rows of up_proj gives 80 tiles,
    more than half of the SMs, so every CTA owns whole 256 x 256 tiles (no split-K) and writes its
    two 128-token MMA halves straight from TMEM. Every row of both halves is checked, with the RMS
    row scale, in bf16 and fp32."""
    from helios_b200 import _lib
    from helios_b200 import quantized as Q
    seed = oracle.matrix_seed(0, 5)
    w, s, b = Q.synth_matrix(seed, 15360, 3840)
    qw = Q.QuantizedWeight.from_mlx(w, s, b, rows=(1280, 3840))
    assert qw.qmm_path(2048) == (_lib.PATH_GEMM, 1)
    x = Q.synth_normal(oracle.activation_seed(2), (2048, 3840))
    xn = u16(x)
    ow, os_, ob = oracle.synth_matrix(seed, 15360, 3840)
    r = np.array([oracle.rms_scale(xn[m]) for m in range(2048)], dtype=np.float32)
    ye, _ = oracle.qmm(xn, ow[1280:3840], os_[1280:3840], ob[1280:3840], row_scale=r)
    yb = Q.quantized_matmul(x, qw, rms_scale=True)
    yg = oracle.bf16_to_f32(u16(yb))
    for h0 in (0, 128):        # token rows of each MMA half of every 256-token tile, separately
        rows = np.concatenate([np.arange(t + h0, t + h0 + 128) for t in range(0, 2048, 256)])
        assert_qmm_close(yg[rows], ye[rows], bf16_out=True)
    yf = Q.quantized_matmul(x, qw, rms_scale=True, out_dtype=torch.float32).cpu().numpy()
    assert_qmm_close(yf, ye, bf16_out=False)
    assert _lib.device_error() == 0
    qw.free()


def test_prefill_gemm_unsplit_full_qkv_2048(cuda, oracle):
    """The full q|k|v projection of one layer (8192 x 3840: q, k and v concatenated as the stack
    uploads them) at 2048 tokens with the RMS row scale: 256 tiles, unsplit."""
    from helios_b200 import _lib
    from helios_b200 import quantized as Q
    mats = [oracle.synth_matrix(oracle.matrix_seed(0, oracle.PROJ_IDS[p]), n, 3840)
            for p, n in (("q", 4096), ("k", 2048), ("v", 2048))]
    dev = [Q.synth_matrix(oracle.matrix_seed(0, oracle.PROJ_IDS[p]), n, 3840) for p, n in (("q", 4096), ("k", 2048),
                                                                                           ("v", 2048))]
    qw = Q.QuantizedWeight.concat([(w, s, b, (0, w.shape[0])) for w, s, b in dev])
    assert qw.rows == 8192 and qw.qmm_path(2048) == (_lib.PATH_GEMM, 1)
    x = Q.synth_normal(oracle.activation_seed(3), (2048, 3840))
    xn = u16(x)
    r = np.array([oracle.rms_scale(xn[m]) for m in range(2048)], dtype=np.float32)
    ow = np.concatenate([m[0] for m in mats])
    os_ = np.concatenate([m[1] for m in mats])
    ob = np.concatenate([m[2] for m in mats])
    ye, _ = oracle.qmm(xn, ow, os_, ob, row_scale=r)
    yb = Q.quantized_matmul(x, qw, rms_scale=True)
    assert_qmm_close(oracle.bf16_to_f32(u16(yb)), ye, bf16_out=True)
    assert _lib.device_error() == 0
    qw.free()


def test_captured_graph_survives_scratch_growth(cuda, oracle):
    """A CUDA graph captured with a decode-width matmul keeps the library scratch it was captured
    with: creating a much larger weight afterwards grows the scratch without freeing the old one,
    so replaying the graph still gives the eager result bit for bit."""
    from helios_b200 import quantized as Q
    N, K = 4096, 3840
    w, s, b = Q.synth_matrix(oracle.matrix_seed(9, 0), N, K)
    qw = Q.QuantizedWeight.from_mlx(w, s, b)
    x = Q.synth_normal(oracle.activation_seed(61), (1, K))
    y = torch.empty((1, N), dtype=torch.bfloat16, device=cuda)
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        Q.quantized_matmul(x, qw, out=y)
    torch.cuda.current_stream().wait_stream(side)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        Q.quantized_matmul(x, qw, out=y)
    # 1,048,576 rows: more stream-K quads than any other weight of the test session
    big = Q.QuantizedWeight.from_mlx(*Q.synth_matrix(oracle.matrix_seed(9, 1), 1 << 20, 64))
    x.copy_(Q.synth_normal(oracle.activation_seed(62), (1, K)))
    g.replay()
    torch.cuda.synchronize()
    eager = Q.quantized_matmul(x, qw)
    assert torch.equal(y, eager)
    del g
    big.free()
    qw.free()


@pytest.mark.parametrize("M", [1, 4])
def test_lm_head_softcap_argmax_full_vocab(cuda, oracle, M):
    from helios_b200 import quantized as Q
    N, K = 262144, 3840
    seed = oracle.matrix_seed(0, 7)
    w, s, b = Q.synth_matrix(seed, N, K)
    qw = Q.QuantizedWeight.from_mlx(w, s, b)
    x = Q.synth_normal(oracle.activation_seed(40 + M), (M, K))
    logits = torch.empty((M, N), dtype=torch.bfloat16, device=cuda)
    tok, val, key = Q.lm_head_argmax(x, qw, softcap=30.0, rms_scale=True, logits=logits)
    xn = u16(x)
    r = np.array([oracle.rms_scale(xn[m]) for m in range(M)], dtype=np.float32)
    ow, os_, ob = oracle.synth_matrix(seed, N, K)
    ye, yb = oracle.qmm(xn, ow, os_, ob, row_scale=r)
    assert_qmm_close(oracle.bf16_to_f32(u16(logits)), ye, bf16_out=True)
    tok, val = tok.cpu().numpy(), val.cpu().numpy()
    for m in range(M):
        # argmax over the GPU's own bf16 logits with the oracle's softcap is exactly what the kernel must return
        t_self, v_self = oracle.softcap_argmax(u16(logits[m]), 30.0)
        assert tok[m] == t_self and val[m] == v_self
        t_ref, v_ref = oracle.softcap_argmax(yb[m], 30.0)
        assert tok[m] == t_ref or abs(v_self - v_ref) <= 0.125, (m, tok[m], t_ref, v_self, v_ref)
    qw.free()


def test_lm_head_row_offset_and_keys(cuda, oracle):
    from helios_b200 import quantized as Q
    from helios_b200.stack import decode_keys
    seed = oracle.matrix_seed(0, 7)
    w, s, b = Q.synth_matrix(seed, 8192, 3840)
    x = Q.synth_normal(oracle.activation_seed(2), (2, 3840))
    halves = [Q.QuantizedWeight.from_mlx(w, s, b, rows=(0, 4096)), Q.QuantizedWeight.from_mlx(w, s, b, rows=(4096, 8192))]
    full = Q.QuantizedWeight.from_mlx(w, s, b)
    tf, vf, kf = Q.lm_head_argmax(x, full)
    keys = [Q.lm_head_argmax(x, h, row_offset=i * 4096)[2].clone() for i, h in enumerate(halves)]
    # combine shards with an unsigned max of the keys (what the TP path does)
    ku = [k.cpu().numpy().view(np.uint64) for k in keys]
    comb = np.maximum(ku[0], ku[1]).view(np.int64)
    t, v = decode_keys(torch.from_numpy(comb))
    assert t == tf.cpu().tolist() and np.allclose(v, vf.cpu().numpy())
    # repeated calls reuse the self-resetting scratch
    tf2, _, _ = Q.lm_head_argmax(x, full)
    assert (tf2 == tf).all()


def test_zero_and_subnormal_scales(cuda, oracle):
    """The decode paths scale s by 2^129 with an exponent add: exact for zero scales (the odd-row
    dequant still returns the bias) and refused by the plan for subnormal ones, which the stream-K
    GEMV sends down its all-magic path instead. Both against the oracle's exact product."""
    from helios_b200 import _lib
    from helios_b200 import quantized as Q
    N, K = 4096, 3840
    w, s, b = oracle.synth_matrix(oracle.matrix_seed(11, 2), N, K)
    x = Q.synth_normal(oracle.activation_seed(77), (1, K))
    s0 = s.copy()
    s0[::7, 3] = 0           # +0.0 scales: q * 0 + b = b for every nibble of those groups
    s0[1::11, 5] = 0x8000    # -0.0
    sub = s0.copy()
    sub[5, 9] = 0x0001       # one subnormal scale

    def upload(scales):
        return Q.QuantizedWeight.from_mlx(torch.from_numpy(w.view(np.int32)).view(torch.uint32),
                                          torch.from_numpy(scales.view(np.int16)).view(torch.bfloat16),
                                          torch.from_numpy(b.view(np.int16)).view(torch.bfloat16))

    for scales, plan_ok in ((s0, True), (sub, False)):
        qw = upload(scales)
        ye, _ = oracle.qmm(u16(x), w, scales, b)
        y = Q.quantized_matmul(x, qw, out_dtype=torch.float32)
        assert_qmm_close(y.cpu().numpy(), ye, bf16_out=False)
        yp = torch.empty((1, N), dtype=torch.bfloat16, device=cuda)
        if plan_ok:
            plan = Q.DecodePlan([(qw, x, yp, 0)], 1)
            plan.run(1)
            torch.cuda.synchronize()
            assert _lib.device_error() == 0
            assert_qmm_close(oracle.bf16_to_f32(u16(yp)), ye, bf16_out=True)
            plan.free()
        else:
            with pytest.raises(_lib.G4qError, match="subnormal"):
                Q.DecodePlan([(qw, x, yp, 0)], 1)
        qw.free()
