"""CPU: the oracle's LoRA delta (add_lora_delta_if_active, native/gemma4_mlx/src/native_model.cc:316-328)
on hand-checkable cases, and the C ABI's argument checks of the LoRA entry points (no GPU needed:
they reject bad arguments before touching the device, with the reference's messages)."""
import ctypes

import numpy as np

from conftest import ROOT  # noqa: F401  (puts the repo root on sys.path)


def bits(vals):
    from oracle import affine
    return affine.f32_to_bf16(np.asarray(vals, dtype=np.float32))


def test_scale_is_alpha_over_rank_rounded_to_bf16(oracle):
    assert oracle.lora_scale_bf16(32.0, 16) == 2.0
    # 1/3 = 0x3EAAAAAB in fp32 -> bf16 0x3EAB (round to nearest even) = 0.333984375
    assert oracle.lora_scale_bf16(1.0, 3) == 0.333984375
    assert oracle.lora_scale_bf16(16.0, 48) == 0.333984375


def test_known_answer_exact(oracle):
    # x = 1..8, A picks x[0] and x[1] -> low = [1, 2]; B = [[1,0],[0,1],[1,1]] -> [1, 2, 3];
    # scale = 4/2 = 2 -> delta = [2, 4, 6]; base [0.5, -4, 1] -> [2.5, 0, 7]
    x = bits([[1, 2, 3, 4, 5, 6, 7, 8]])
    a = np.zeros((2, 8), np.float32)
    a[0, 0] = a[1, 1] = 1.0
    b = np.array([[1, 0], [0, 1], [1, 1]], np.float32)
    y = oracle.lora_delta(x, bits([[0.5, -4.0, 1.0]]), a, b, alpha=4.0)
    assert oracle.bf16_to_f32(y).tolist() == [[2.5, 0.0, 7.0]]


def test_two_bf16_roundings(oracle):
    # delta = 1 + 2^-9 rounds to 1 in bf16 (tie to even) before the add; 256 + 1 = 257 rounds to 256
    x = bits([[1, 0, 0, 0, 0, 0, 0, 0]])
    a = np.zeros((1, 8), np.float32)
    a[0, 0] = 1.0
    b = np.array([[1.0 + 2.0 ** -9], [1.0]], np.float32)
    y = oracle.lora_delta(x, bits([[0.0, 256.0]]), a, b, alpha=1.0)
    assert oracle.bf16_to_f32(y).tolist() == [[1.0, 256.0]]
    # rank 3, alpha 1: the scale is bf16(1/3) = 0.333984375, not 1/3: 3.5 * 0.333984375 = 1.16894...
    # rounds to 1.171875 in bf16, where 3.5 / 3 = 1.16666... would round to 1.1640625
    a3 = np.zeros((3, 8), np.float32)
    a3[0, 0] = 1.0
    b3 = np.array([[3.5, 0.0, 0.0]], np.float32)
    y3 = oracle.lora_delta(x, bits([[0.0]]), a3, b3, alpha=1.0)
    assert oracle.bf16_to_f32(y3)[0, 0] == 1.171875


def test_lora_create_rejects_bad_arguments_without_gpu():
    from helios_b200 import _lib
    L = _lib.load()
    h = ctypes.c_void_p()
    a = (ctypes.c_float * 64)()
    assert L.g4q_lora_create(8, 8, 0, 1.0, a, a, 1, ctypes.byref(h)) == _lib.G4Q_ERR_INVALID_ARGUMENT
    assert "rank must be greater than zero" in _lib.last_error()
    for alpha in (0.0, -1.0, float("inf"), float("nan")):
        assert L.g4q_lora_create(8, 8, 4, alpha, a, a, 1, ctypes.byref(h)) == _lib.G4Q_ERR_INVALID_ARGUMENT
        assert "alpha must be finite and positive" in _lib.last_error()
    assert L.g4q_lora_create(8, 12, 4, 1.0, a, a, 1, ctypes.byref(h)) == _lib.G4Q_ERR_INVALID_ARGUMENT
    assert L.g4q_lora_create(8, 8, 257, 1.0, a, a, 1, ctypes.byref(h)) == _lib.G4Q_ERR_UNSUPPORTED_CONFIG
    assert L.g4q_lora_create(8, 8, 4, 1.0, a, a, 0, ctypes.byref(h)) == _lib.G4Q_ERR_INVALID_ARGUMENT
    assert not h
    assert L.g4q_lora_apply(None, None, 1, 8, None, 8, None) == _lib.G4Q_ERR_INVALID_ARGUMENT
    assert "LoRA handle" in _lib.last_error()
    bogus = ctypes.create_string_buffer(256)
    assert L.g4q_lora_free(ctypes.cast(bogus, ctypes.c_void_p)) == _lib.G4Q_ERR_INVALID_ARGUMENT
    assert "invalid LoRA handle" in _lib.last_error()
