"""GPU: the MLP's elementwise neighbours against the CPU oracle, through the C ABI, and the real
model's MLP block built from them (rms_norm -> gate|up quantized matmul -> geglu -> down quantized
matmul, native/gemma4_mlx/src/native_model.cc:929-949).

geglu and rms_norm repeat the reference's bf16 roundings op for op; what can differ is the last
fp32 bit of tanh (CUDA's tanhf against numpy's) and of the RMSNorm's sum of squares (another
summation order), which flips a bf16 rounding only next to a rounding boundary. Checked: at
least 99.9 % (geglu) / 99 % (rms_norm) of the outputs bit-identical, the rest within one bf16 ulp.
The MLP block is checked with the matmul tolerance, max|y - y_oracle| <= 1e-2 * rms(y_oracle)."""
import numpy as np
import pytest
import torch

from gpu_util import assert_qmm_close, dev_u16, u16, u32

pytestmark = pytest.mark.gpu


def ulps_apart(oracle, a, b):
    fa = oracle.bf16_to_f32(a).astype(np.float64)
    fb = oracle.bf16_to_f32(b).astype(np.float64)
    ulp = 2.0 ** (np.floor(np.log2(np.maximum(np.abs(fb), 2.0 ** -126))) - 7)
    return np.abs(fa - fb) / ulp


def test_geglu_matches_oracle_on_gate_up_halves(cuda, oracle):
    from helios_b200 import quantized as Q
    M, I = 5, 15360
    g = torch.Generator().manual_seed(1)
    y = (2.0 * torch.randn(M, 2 * I, generator=g)).to(torch.bfloat16).to(cuda)   # one gate|up output
    act = Q.geglu(y[:, :I], y[:, I:])
    torch.cuda.synchronize()
    ref = oracle.geglu(u16(y)[:, :I], u16(y)[:, I:])
    got = u16(act)
    assert (got == ref).mean() >= 0.999, (got == ref).mean()
    assert ulps_apart(oracle, got, ref).max() <= 1.0


def test_geglu_edge_values(cuda, oracle):
    from helios_b200 import quantized as Q
    vals = np.array([0.0, -0.0, 1.0, -1.0, 4.0, -4.0, 30.0, -30.0, 1e-30, -1e-30, 0.5, -0.5, 100.0, -100.0,
                     2.0 ** -130, 3.0], np.float32)
    gate = oracle.f32_to_bf16(np.tile(vals, 8).reshape(8, 16))
    up = oracle.f32_to_bf16(np.full((8, 16), 1.5, np.float32))
    got = u16(Q.geglu(dev_u16(gate, cuda), dev_u16(up, cuda)))
    ref = oracle.geglu(gate, up)
    assert (got == ref).all(), (oracle.bf16_to_f32(got), oracle.bf16_to_f32(ref))


@pytest.mark.parametrize("with_weight", [True, False])
def test_rms_norm_matches_oracle(cuda, oracle, with_weight):
    from helios_b200 import quantized as Q
    M, K = 7, 3840
    g = torch.Generator().manual_seed(2)
    x = (3.0 * torch.randn(M, K, generator=g)).to(torch.bfloat16).to(cuda)
    w = (1.0 + 0.2 * torch.randn(K, generator=g)).to(torch.bfloat16).to(cuda) if with_weight else None
    out = Q.rms_norm(x, w, 1e-6)
    torch.cuda.synchronize()
    ref = oracle.rms_norm(u16(x), None if w is None else u16(w), 1e-6)
    got = u16(out)
    assert (got == ref).mean() >= 0.99, (got == ref).mean()
    assert ulps_apart(oracle, got, ref).max() <= 1.0
    # in place gives the same bits
    x2 = x.clone()
    Q.rms_norm(x2, w, 1e-6, out=x2)
    assert (u16(x2) == got).all()


def test_real_mlp_block(cuda, oracle):
    """h -> rms_norm(pre_feedforward_layernorm) -> gate|up (one concatenated 4-bit matmul) ->
    geglu -> down, at the real model's shapes (3840 -> 2 x 15360 -> 3840), two tokens."""
    from helios_b200 import quantized as Q
    M, H, I = 2, 3840, 15360
    gw = Q.synth_matrix(oracle.matrix_seed(3, oracle.PROJ_IDS["gate"]), I, H, device=cuda)
    uw = Q.synth_matrix(oracle.matrix_seed(3, oracle.PROJ_IDS["up"]), I, H, device=cuda)
    dw = Q.synth_matrix(oracle.matrix_seed(3, oracle.PROJ_IDS["down"]), H, I, device=cuda)
    gate_up = Q.QuantizedWeight.concat([gw, uw])
    down = Q.QuantizedWeight.from_mlx(*dw)
    g = torch.Generator().manual_seed(3)
    h = (2.0 * torch.randn(M, H, generator=g)).to(torch.bfloat16).to(cuda)
    norm_w = (1.0 + 0.1 * torch.randn(H, generator=g)).to(torch.bfloat16).to(cuda)

    hn = Q.rms_norm(h, norm_w, 1e-6)
    gu = Q.quantized_matmul(hn, gate_up)
    act = Q.geglu(gu[:, :I], gu[:, I:])
    y = Q.quantized_matmul(act, down)
    torch.cuda.synchronize()

    # the oracle's chain on the same inputs
    ogw, ouw, odw = ((u32(w), u16(s), u16(b)) for w, s, b in (gw, uw, dw))
    hn_ref = oracle.rms_norm(u16(h), u16(norm_w), 1e-6)
    _, gate_ref = oracle.qmm(hn_ref, *ogw)
    _, up_ref = oracle.qmm(hn_ref, *ouw)
    act_ref = oracle.geglu(gate_ref, up_ref)
    y_exact, y_ref = oracle.qmm(act_ref, *odw)
    got = oracle.bf16_to_f32(u16(y)).astype(np.float64)
    rms = float(np.sqrt(np.mean(y_exact ** 2)))
    assert np.abs(got - oracle.bf16_to_f32(y_ref)).max() <= 1e-2 * rms
    assert (u16(act) == act_ref).mean() >= 0.99
    gate_up.free()
    down.free()


@pytest.mark.parametrize("proj,N,K", [("gate_up", 30720, 3840), ("down", 3840, 15360), ("qkv", 8192, 3840)])
@pytest.mark.parametrize("M", [1, 2, 4, 8])
def test_norm_fused_into_decode_gemv(cuda, oracle, proj, N, K, M):
    """rms_norm -> quantized matmul as one stream-K GEMV launch (the norm applied while x is staged;
    down_proj's K = 15360 exercises the staged window of x, at 8 tokens with 12 warps per CTA) against
    the oracle's two steps."""
    from helios_b200 import quantized as Q
    seed = oracle.matrix_seed(7, oracle.PROJ_IDS["up" if proj != "down" else "down"])
    w, s, b = Q.synth_matrix(seed, N, K)
    qw = Q.QuantizedWeight.from_mlx(w, s, b)
    g = torch.Generator().manual_seed(M + K)
    x = (2.0 * torch.randn(M, K, generator=g)).to(torch.bfloat16).to(cuda)
    nw = (1.0 + 0.2 * torch.randn(K, generator=g)).to(torch.bfloat16).to(cuda)
    xn = torch.empty_like(x)
    y = Q.norm_quantized_matmul(x, nw, qw, eps=1e-6, xn=xn)
    y2 = Q.norm_quantized_matmul(x, nw, qw, eps=1e-6)      # without the normalized-rows output
    torch.cuda.synchronize()
    xn_ref = oracle.rms_norm(u16(x), u16(nw), 1e-6)
    assert (u16(xn) == xn_ref).mean() >= 0.99 and ulps_apart(oracle, u16(xn), xn_ref).max() <= 1.0
    ow, os_, ob = u32(w), u16(s), u16(b)
    # the matmul consumed exactly the normalized rows it wrote out
    ye, yb = oracle.qmm(u16(xn), ow, os_, ob)
    assert_qmm_close(oracle.bf16_to_f32(u16(y)), ye, bf16_out=True)
    assert (u16(y) == yb).mean() > 0.99
    assert (u16(y2) == u16(y)).all()
    # and the whole pair is within the matmul tolerance of the oracle's rms_norm -> qmm
    ye2, _ = oracle.qmm(xn_ref, ow, os_, ob)
    assert_qmm_close(oracle.bf16_to_f32(u16(y)), ye2, bf16_out=True)
    qw.free()


@pytest.mark.parametrize("M", [12, 64])
def test_norm_matmul_outside_the_fused_widths(cuda, oracle, M):
    """M > 8: the normalized rows go through xn (required) and the regular matmul path."""
    from helios_b200 import _lib
    from helios_b200 import quantized as Q
    N, K = 2048, 3840
    seed = oracle.matrix_seed(8, oracle.PROJ_IDS["k"])
    w, s, b = Q.synth_matrix(seed, N, K)
    qw = Q.QuantizedWeight.from_mlx(w, s, b)
    g = torch.Generator().manual_seed(M)
    x = (2.0 * torch.randn(M, K, generator=g)).to(torch.bfloat16).to(cuda)
    nw = (1.0 + 0.2 * torch.randn(K, generator=g)).to(torch.bfloat16).to(cuda)
    with pytest.raises(_lib.G4qInvalidArgument):
        Q.norm_quantized_matmul(x, nw, qw)
    xn = torch.empty_like(x)
    y = Q.norm_quantized_matmul(x, nw, qw, xn=xn)
    torch.cuda.synchronize()
    xn_ref = oracle.rms_norm(u16(x), u16(nw), 1e-6)
    assert (u16(xn) == xn_ref).mean() >= 0.99
    ye, _ = oracle.qmm(xn_ref, u32(w), u16(s), u16(b))
    assert_qmm_close(oracle.bf16_to_f32(u16(y)), ye, bf16_out=True)
    qw.free()


def _pair_case(oracle, cuda, M, I=15360, K=3840, layer=9):
    from helios_b200 import quantized as Q
    gw = Q.synth_matrix(oracle.matrix_seed(layer, oracle.PROJ_IDS["gate"]), I, K, device=cuda)
    uw = Q.synth_matrix(oracle.matrix_seed(layer, oracle.PROJ_IDS["up"]), I, K, device=cuda)
    pair = Q.QuantizedWeight.geglu_pair(gw, uw)
    x = Q.synth_normal(oracle.activation_seed(60 + M), (M, K), device=cuda)
    return Q, gw, uw, pair, x


@pytest.mark.parametrize("M", [1, 2, 4, 8])
@pytest.mark.parametrize("rms", [False, True])
def test_geglu_fused_into_decode_gemv(cuda, oracle, M, rms):
    """gate|up matmul + GeGLU as one stream-K GEMV launch: bit-identical to the paired matmul followed
    by the GeGLU kernel, and within the matmul tolerance of the oracle's gate, up and geglu."""
    Q, gw, uw, pair, x = _pair_case(oracle, cuda, M)
    I = gw[0].shape[0]
    act = Q.quantized_matmul_geglu(x, pair, rms_scale=rms)
    y = Q.quantized_matmul(x, pair, rms_scale=rms)                   # [M, 2I], paired order
    yp = y.view(M * I // 32, 64)
    act2 = Q.geglu(yp[:, :32], yp[:, 32:]).view(M, I)
    torch.cuda.synchronize()
    assert (u16(act) == u16(act2)).all()
    if not rms:
        _, gate_ref = oracle.qmm(u16(x), u32(gw[0]), u16(gw[1]), u16(gw[2]))
        _, up_ref = oracle.qmm(u16(x), u32(uw[0]), u16(uw[1]), u16(uw[2]))
        ref = oracle.geglu(gate_ref, up_ref)
        got = u16(act)
        assert (got == ref).mean() > 0.99
        gf, rf = oracle.bf16_to_f32(got).astype(np.float64), oracle.bf16_to_f32(ref).astype(np.float64)
        assert np.abs(gf - rf).max() <= 1e-2 * float(np.sqrt(np.mean(rf ** 2))) + np.abs(rf).max() * 2.0 ** -8
    pair.free()


@pytest.mark.parametrize("M,I,K,splits", [(40, 2048, 1024, 4), (2048, 15360, 3840, 1), (2048, 256, 3840, 8),
                                          (300, 7680, 3840, 1)])
@pytest.mark.parametrize("rms", [False, True])
def test_geglu_fused_into_prefill_gemm(cuda, oracle, M, I, K, splits, rms):
    """gate|up matmul + GeGLU at prefill widths in the tcgen05 GEMM's epilogue (unsplit tiles) or in its
    split-K reduction (small I): bit-identical to the paired matmul followed by the GeGLU kernel, and
    within the matmul tolerance of the oracle's gate, up and geglu (checked without the RMS scale)."""
    from helios_b200 import _lib
    Q, gw, uw, pair, x = _pair_case(oracle, cuda, M, I=I, K=K, layer=12)
    assert pair.qmm_path(M) == (_lib.PATH_GEMM, splits)
    act = Q.quantized_matmul_geglu(x, pair, rms_scale=rms)
    y = Q.quantized_matmul(x, pair, rms_scale=rms)
    yp = y.view(M * I // 32, 64)
    act2 = Q.geglu(yp[:, :32], yp[:, 32:]).view(M, I)
    torch.cuda.synchronize()
    assert (u16(act) == u16(act2)).all()
    assert _lib.device_error() == 0
    if not rms and M <= 300:
        # gate and up within the matmul tolerance of the oracle's exact products, and the GeGLU the
        # oracle's nine bf16 steps on exactly those gate / up values (a one-ulp flip of gate or up is
        # within the matmul tolerance but moves gelu * up by an ulp of the product, so the GeGLU is
        # compared on the GPU's own gate and up)
        yg = u16(y).reshape(M, I // 32, 64)
        gate_gpu = np.ascontiguousarray(yg[:, :, :32].reshape(M, I))
        up_gpu = np.ascontiguousarray(yg[:, :, 32:].reshape(M, I))
        ge, _ = oracle.qmm(u16(x), u32(gw[0]), u16(gw[1]), u16(gw[2]))
        ue, _ = oracle.qmm(u16(x), u32(uw[0]), u16(uw[1]), u16(uw[2]))
        assert_qmm_close(oracle.bf16_to_f32(gate_gpu), ge, bf16_out=True)
        assert_qmm_close(oracle.bf16_to_f32(up_gpu), ue, bf16_out=True)
        ref = oracle.geglu(gate_gpu, up_gpu)
        got = u16(act)
        assert (got == ref).mean() > 0.999 and ulps_apart(oracle, got, ref).max() <= 1.0
    pair.free()


@pytest.mark.parametrize("M", [12, 16])
def test_geglu_pair_outside_the_fused_widths(cuda, oracle, M):
    """9 <= M <= 16 (the cluster GEMV): the paired matmul output goes through y (required), then the
    GeGLU kernel."""
    from helios_b200 import _lib
    Q, gw, uw, pair, x = _pair_case(oracle, cuda, M, I=2048, K=1024, layer=10)
    I = 2048
    with pytest.raises(_lib.G4qInvalidArgument):
        Q.quantized_matmul_geglu(x, pair)
    y = torch.empty((M, 2 * I), dtype=torch.bfloat16, device=cuda)
    act = Q.quantized_matmul_geglu(x, pair, y=y)
    yref = Q.quantized_matmul(x, pair)
    yp = yref.view(M * I // 32, 64)
    act2 = Q.geglu(yp[:, :32], yp[:, 32:]).view(M, I)
    torch.cuda.synchronize()
    assert (u16(y) == u16(yref)).all() and (u16(act) == u16(act2)).all()
    pair.free()


@pytest.mark.parametrize("M", [1, 4, 8])
def test_norm_gate_up_geglu_in_one_launch(cuda, oracle, M):
    """pre_feedforward_layernorm -> gate|up -> geglu (native_model.cc:929-945) as one GEMV launch:
    bit-identical to norm_quantized_matmul (the same fused norm) followed by the GeGLU kernel."""
    from helios_b200 import _lib
    Q, gw, uw, pair, x = _pair_case(oracle, cuda, M, layer=11)
    I, K = gw[0].shape[0], x.shape[1]
    g = torch.Generator().manual_seed(70 + M)
    nw = (1.0 + 0.2 * torch.randn(K, generator=g)).to(torch.bfloat16).to(cuda)
    act = Q.quantized_matmul_geglu(x, pair, norm_weight=nw)
    y = Q.norm_quantized_matmul(x, nw, pair)
    yp = y.view(M * I // 32, 64)
    act2 = Q.geglu(yp[:, :32], yp[:, 32:]).view(M, I)
    torch.cuda.synchronize()
    assert (u16(act) == u16(act2)).all()
    with pytest.raises(_lib.G4qInvalidArgument):
        Q.quantized_matmul_geglu(x, pair, norm_weight=nw, rms_scale=True)
    pair.free()


@pytest.mark.parametrize("with_scalar", [True, False])
def test_rms_norm_residual_layer_scalar(cuda, oracle, with_scalar):
    """post_feedforward_layernorm -> residual add -> layer_scalar (native_model.cc:954-968) in one
    kernel, in place on the residual stream, against the oracle's three rounded steps."""
    from helios_b200 import quantized as Q
    M, K = 5, 3840
    g = torch.Generator().manual_seed(80)
    x = (3.0 * torch.randn(M, K, generator=g)).to(torch.bfloat16).to(cuda)
    w = (1.0 + 0.2 * torch.randn(K, generator=g)).to(torch.bfloat16).to(cuda)
    res = (4.0 * torch.randn(M, K, generator=g)).to(torch.bfloat16).to(cuda)
    sc = torch.tensor([0.71875], dtype=torch.bfloat16, device=cuda) if with_scalar else None
    r0 = u16(res).copy()
    Q.rms_norm_residual(x, w, res, sc, 1e-6, out=res)
    torch.cuda.synchronize()
    ref = oracle.rms_norm_residual(u16(x), u16(w), r0, None if sc is None else int(u16(sc)[0]), 1e-6)
    got = u16(res)
    assert (got == ref).mean() >= 0.99, (got == ref).mean()
    assert ulps_apart(oracle, got, ref).max() <= 1.0
