"""GPU: quantization specs other than 4-bit / group 64: the 8-bit group-64 per-module override a
model's manifest may name, and groups 32 / 128 as mlx::core accepts them. Those weights stay in
MLX's layout on the device and run on the generic kernels; results are checked against the CPU
oracle through the C ABI: dequantize bit-exact (full matrix and gathered rows, both rounding chains), quantized matmul
within max|y - y_oracle| <= 1e-2 * rms(y_oracle) (bf16 output rounding excluded, as for the
4-bit path)."""
import numpy as np
import pytest
import torch

from gpu_util import assert_qmm_close, dev_u16, dev_u32, u16, u32

pytestmark = pytest.mark.gpu

SPECS = [(8, 64), (8, 32), (8, 128), (4, 32), (4, 128)]


def upload(Q, cuda, w, s, b, bits, gs, **kw):
    return Q.QuantizedWeight.from_mlx(dev_u32(w, cuda), dev_u16(s, cuda), dev_u16(b, cuda), bits=bits,
                                      group_size=gs, **kw)


@pytest.mark.parametrize("bits,gs", SPECS)
def test_dequantize_bit_exact(cuda, oracle, bits, gs):
    from helios_b200 import quantized as Q
    N, K = 72, 768
    w, s, b = oracle.synth_matrix(1000 + bits * gs, N, K, bits=bits, group_size=gs)
    q = upload(Q, cuda, w, s, b, bits, gs)
    assert q.info()["bits"] == bits and q.info()["group_size"] == gs
    for chain in (Q.CHAIN_R2, Q.CHAIN_R1):
        ref = oracle.dequantize(w, s, b, bits=bits, group_size=gs, chain=chain)
        assert (u16(Q.dequantize(q, bits=bits, group_size=gs, chain=chain)) == ref).all()
        # the same op straight from MLX-layout device tensors
        d = Q.dequantize(dev_u32(w, cuda), dev_u16(s, cuda), dev_u16(b, cuda), group_size=gs, bits=bits, chain=chain)
        assert (u16(d) == ref).all()
    ids = np.array([5, 0, 71, 5, 33], dtype=np.int32)
    g = Q.dequantize(q, bits=bits, group_size=gs, rows=torch.from_numpy(ids))
    assert (u16(g) == oracle.dequantize_rows(w, s, b, ids, bits=bits, group_size=gs)).all()
    assert q.info()["error_flags"] == 0
    q.free()


def test_gather_out_of_range_ids(cuda, oracle):
    """An id outside [0, rows) gives a zero row and raises bit 2 of the handle's error flags."""
    from helios_b200 import quantized as Q
    w, s, b = oracle.synth_matrix(7, 48, 256, bits=8, group_size=32)
    q = upload(Q, cuda, w, s, b, 8, 32)
    ids = np.array([3, -1, 48, 47], dtype=np.int32)
    g = u16(Q.dequantize(q, bits=8, group_size=32, rows=torch.from_numpy(ids)))
    ok = oracle.dequantize_rows(w, s, b, np.array([3, 47], dtype=np.int32), bits=8, group_size=32)
    assert (g[0] == ok[0]).all() and (g[3] == ok[1]).all()
    assert (g[1] == 0).all() and (g[2] == 0).all()
    assert q.info()["error_flags"] == 2
    q.free()


@pytest.mark.parametrize("bits,gs", SPECS)
@pytest.mark.parametrize("M", [1, 3, 17])
def test_qmm_against_oracle(cuda, oracle, bits, gs, M):
    from helios_b200 import quantized as Q
    N, K = 1040, 3840
    w, s, b = oracle.synth_matrix(oracle.matrix_seed(9, bits + gs), N, K, bits=bits, group_size=gs)
    x = oracle.synth_normal_bf16(oracle.activation_seed(M + gs), M * K).reshape(M, K)
    q = upload(Q, cuda, w, s, b, bits, gs)
    ye, yb = oracle.qmm(x, w, s, b, bits=bits, group_size=gs)
    y = Q.quantized_matmul(dev_u16(x, cuda), q, group_size=gs, bits=bits)
    assert y.shape == (M, N) and y.dtype == torch.bfloat16
    assert_qmm_close(oracle.bf16_to_f32(u16(y)), ye, bf16_out=True)
    yf = Q.quantized_matmul(dev_u16(x, cuda), q, group_size=gs, bits=bits, out_dtype=torch.float32)
    assert_qmm_close(yf.cpu().numpy(), ye, bf16_out=False)
    q.free()


def test_qmm_rms_scale_strided_and_per_call_upload(cuda, oracle):
    """RMS_SCALE folds 1/sqrt(mean(x^2)+eps) into the output; x may be a strided view; MLX-layout
    tensors passed straight to quantized_matmul are uploaded for the call."""
    from helios_b200 import quantized as Q
    M, N, K, eps = 5, 200, 1024, 1e-6
    w, s, b = oracle.synth_matrix(321, N, K, bits=8, group_size=128)
    x = oracle.synth_normal_bf16(17, M * (K + 64)).reshape(M, K + 64)
    xs = x[:, 32:32 + K]
    rs = np.array([oracle.rms_scale(r, eps) for r in xs], dtype=np.float32)
    ye, _ = oracle.qmm(xs, w, s, b, bits=8, group_size=128, row_scale=rs)
    xd = dev_u16(x, cuda)[:, 32:32 + K]
    q = upload(Q, cuda, w, s, b, 8, 128)
    yf = Q.quantized_matmul(xd, q, group_size=128, bits=8, rms_scale=True, eps=eps, out_dtype=torch.float32)
    assert_qmm_close(yf.cpu().numpy(), ye, bf16_out=False)
    ye0, _ = oracle.qmm(xs, w, s, b, bits=8, group_size=128)
    y0 = Q.quantized_matmul(xd, dev_u32(w, cuda), dev_u16(s, cuda), dev_u16(b, cuda), group_size=128, bits=8,
                            out_dtype=torch.float32)
    assert_qmm_close(y0.cpu().numpy(), ye0, bf16_out=False)
    q.free()


def test_windows_concat_export(cuda, oracle):
    """Row windows (column split), group-aligned column windows (row split), concatenation and the
    export round trip keep every byte of the MLX arrays; host and device sources load alike."""
    from helios_b200 import quantized as Q
    bits, gs, N, K = 8, 32, 96, 512
    w, s, b = oracle.synth_matrix(55, N, K, bits=bits, group_size=gs)
    full = oracle.dequantize(w, s, b, bits=bits, group_size=gs)
    per = 32 // bits
    q = upload(Q, cuda, w, s, b, bits, gs, rows=(24, 72), cols=(128, 384))
    assert q.shape == (48, 256)
    assert (u16(Q.dequantize(q, bits=bits, group_size=gs)) == full[24:72, 128:384]).all()
    ew, es, eb = q.export()
    assert (u32(ew) == w[24:72, 128 // per:384 // per]).all()
    assert (u16(es) == s[24:72, 128 // gs:384 // gs]).all() and (u16(eb) == b[24:72, 128 // gs:384 // gs]).all()
    q.free()
    w2, s2, b2 = oracle.synth_matrix(56, 40, K, bits=bits, group_size=gs)
    host = lambda a, t: torch.from_numpy(a.view(np.int32 if t == torch.uint32 else np.int16)).view(t)
    c = Q.QuantizedWeight.concat([(dev_u32(w, cuda), dev_u16(s, cuda), dev_u16(b, cuda), (0, 16)),
                                  (host(w2, torch.uint32), host(s2, torch.bfloat16), host(b2, torch.bfloat16))],
                                 bits=bits, group_size=gs)
    d = u16(Q.dequantize(c, bits=bits, group_size=gs))
    assert (d[:16] == full[:16]).all()
    assert (d[16:] == oracle.dequantize(w2, s2, b2, bits=bits, group_size=gs)).all()
    with pytest.raises(Exception):
        upload(Q, cuda, w, s, b, bits, gs, cols=(16, 272))   # column window not group aligned
    c.free()


def test_fused_paths_take_only_the_kernel_layout(cuda, oracle):
    """The fused LM head and the persistent decode plan run on 4-bit group-64 weights only; other
    specs get a clear status instead of a wrong answer."""
    from helios_b200 import _lib
    from helios_b200 import quantized as Q
    w, s, b = oracle.synth_matrix(3, 64, 256, bits=8, group_size=64)
    q = upload(Q, cuda, w, s, b, 8, 64)
    x = torch.zeros((1, 256), dtype=torch.bfloat16, device=cuda)
    y = torch.zeros((1, 64), dtype=torch.bfloat16, device=cuda)
    with pytest.raises(_lib.G4qError) as e:
        Q.lm_head_argmax(x, q)
    assert e.value.status == _lib.G4Q_ERR_UNSUPPORTED_CONFIG
    with pytest.raises(_lib.G4qError) as e:
        Q.DecodePlan([(q, x, y, 0)])
    assert e.value.status == _lib.G4Q_ERR_UNSUPPORTED_CONFIG
    q.free()
