"""CPU: the oracle's GeGLU (native/gemma4_mlx/src/native_model.cc:378-386) and RMSNorm
(fast::rms_norm as called at :910-913) on hand-computed cases, and the C ABI's argument checks
of g4q_geglu / g4q_rms_norm (rejected before any device work, so no GPU is needed)."""
import ctypes

import numpy as np

from conftest import ROOT  # noqa: F401  (puts the repo root on sys.path)


def b16(oracle, vals):
    return oracle.f32_to_bf16(np.asarray(vals, dtype=np.float32))


def test_geglu_known_answers(oracle):
    # By hand, every op rounded to bf16 (constants bf16(0.044715) = 0.044677734375,
    # bf16(0.79788456) = 0.796875):
    #   g = 1: g + 0.0446777 = 1.0446777 -> 1.046875; * 0.796875 = 0.8342285 -> 0.8359375;
    #          tanh -> 0.68365 -> 0.68359375; 1 + t = 1.68359375 -> 1.6875 (tie to even);
    #          0.5 * 1.6875 = 0.84375
    #   g = 4: 4 + 2.859375 = 6.859375 -> 6.875 (tie to even); * 0.796875 -> 5.46875;
    #          tanh -> 0.99996 -> 1.0; gelu = 2 * 2 = 4; * 1.5 = 6
    #   g = -4: tanh -> -1.0, 1 + t = 0, gelu = -2 * 0 = -0.0
    out = oracle.geglu(b16(oracle, [1, 4, -4, 0]), b16(oracle, [1, 1.5, 1.5, 3]))
    assert oracle.bf16_to_f32(out).tolist() == [0.84375, 6.0, -0.0, 0.0]
    assert int(out[2]) == 0x8000


def test_geglu_rounds_every_op(oracle):
    # one rounding at the end (fp32 GELU, then bf16) differs from the nine roundings on some inputs
    rng = np.random.default_rng(0)
    g = b16(oracle, rng.normal(0, 2, 4096))
    u = b16(oracle, np.ones(4096))
    nine = oracle.geglu(g, u)
    gf = oracle.bf16_to_f32(g).astype(np.float64)
    once = oracle.f32_to_bf16((0.5 * gf * (1 + np.tanh(0.7978845608028654 * (gf + 0.044715 * gf ** 3)))).astype(np.float32))
    assert (nine != once).any()
    assert np.abs(oracle.bf16_to_f32(nine) - oracle.bf16_to_f32(once)).max() < 0.1


def test_rms_norm_known_answers(oracle):
    x = b16(oracle, [[2] * 8, [1] * 8, [3, 4, 0, 0, 0, 0, 0, 0]])
    w = b16(oracle, [2] * 8)
    out = oracle.bf16_to_f32(oracle.rms_norm(x, w, eps=0.0))
    assert out[0].tolist() == [2.0] * 8 and out[1].tolist() == [2.0] * 8
    # rms of [3, 4, 0 x 6] = sqrt(25 / 8): 3 / 1.7677670 = 1.6970563 -> bf16 1.6953125, then x 2
    assert out[2, :2].tolist() == [3.390625, 4.53125]
    assert oracle.bf16_to_f32(oracle.rms_norm(x[2:], None, eps=0.0))[0, :2].tolist() == [1.6953125, 2.265625]


def test_mlp_entry_points_reject_bad_arguments_without_gpu():
    from helios_b200 import _lib
    L = _lib.load()
    buf = ctypes.create_string_buffer(64)
    p = ctypes.cast(buf, ctypes.c_void_p)
    assert L.g4q_geglu(p, 8, p, 8, 1, 12, p, 8, None) == _lib.G4Q_ERR_INVALID_ARGUMENT
    assert "multiple of 8" in _lib.last_error()
    assert L.g4q_geglu(None, 8, p, 8, 1, 8, p, 8, None) == _lib.G4Q_ERR_INVALID_ARGUMENT
    assert L.g4q_geglu(p, 4, p, 8, 1, 8, p, 8, None) == _lib.G4Q_ERR_INVALID_ARGUMENT
    assert "strides" in _lib.last_error()
    assert L.g4q_geglu(p, 8, p, 8, 0, 8, p, 8, None) == _lib.G4Q_OK       # nothing to do
    assert L.g4q_rms_norm(p, 8, None, 1, 12, 1e-6, p, 8, None) == _lib.G4Q_ERR_INVALID_ARGUMENT
    assert L.g4q_rms_norm(p, 8, None, 1, 8, float("nan"), p, 8, None) == _lib.G4Q_ERR_INVALID_ARGUMENT
    assert "eps" in _lib.last_error()
    assert L.g4q_rms_norm(None, 8, None, 1, 8, 1e-6, p, 8, None) == _lib.G4Q_ERR_INVALID_ARGUMENT


def test_fused_matmul_entry_points_reject_bad_arguments_without_gpu():
    from helios_b200 import _lib
    L = _lib.load()
    buf = ctypes.create_string_buffer(64)
    p = ctypes.cast(buf, ctypes.c_void_p)
    assert L.g4q_qmm_norm(None, p, 1, 8, p, 1e-6, None, 0, p, 8, None) == _lib.G4Q_ERR_INVALID_ARGUMENT
    assert "weight handle" in _lib.last_error()
    assert L.g4q_qmm_geglu(None, p, 1, 8, None, 0, 1e-6, None, p, 8, None) == _lib.G4Q_ERR_INVALID_ARGUMENT
    assert "weight handle" in _lib.last_error()
    assert L.g4q_qmm_geglu(p, p, 1, 8, None, 0, 1e-6, None, p, 8, None) == _lib.G4Q_ERR_INVALID_ARGUMENT
    assert "invalid weight handle" in _lib.last_error()


def test_rms_norm_residual_known_answer(oracle):
    # the norm of [2]*8 with weight 2 and eps 0 is 2; residual 256 + 2 = 258 (exact in bf16);
    # x 1.5 = 387 lies halfway between the bf16 neighbours 386 and 388: ties to even -> 388
    x = b16(oracle, [[2] * 8])
    w = b16(oracle, [2] * 8)
    r = b16(oracle, [[256] * 8])
    out = oracle.rms_norm_residual(x, w, r, int(b16(oracle, [1.5])[0]), eps=0.0)
    assert oracle.bf16_to_f32(out)[0].tolist() == [388.0] * 8
    # without a scalar: 256 + 2 = 258 (exact in bf16)
    assert oracle.bf16_to_f32(oracle.rms_norm_residual(x, w, r, None, eps=0.0))[0].tolist() == [258.0] * 8
