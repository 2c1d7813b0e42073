"""GPU: the allocation-free LM head (g4q_lm_head_argmax_noalloc) against the regular entry point.

Some callers cannot allocate device memory when they call the library: code running inside a CUDA
stream capture (cudaMalloc is not allowed there) and host runtimes that own every device byte
through a pre-sized arena. For them the allocation-free entry point takes the weight in kernel
layout v1 in caller-owned memory and keeps its small argmax scratch in a static array inside the
library. This test calls it through the C ABI twice in a row and checks tokens, values, keys and
logits against g4q_lm_head_argmax on the same weights and inputs. It lives in its own file,
collected last, and passes alone in a fresh process as well as after the other tests.
"""
import ctypes

import numpy as np
import pytest
import torch

from gpu_util import assert_qmm_close, u16

pytestmark = pytest.mark.gpu


def _p(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


@pytest.mark.parametrize("M", [1, 5])
def test_noalloc_lm_head_matches_regular_entry_point(cuda, oracle, M):
    from helios_b200 import _lib
    from helios_b200 import quantized as Q
    N, K = 32768, 3840
    seed = oracle.matrix_seed(0, 7)
    w, s, b = oracle.synth_matrix(seed, N, K)
    # the weight in kernel layout v1, in memory the caller owns (here: torch tensors)
    packed, sb = oracle.repack(w, s, b)
    d_packed = torch.from_numpy(packed.view(np.int32)).to(cuda)
    d_sb = torch.from_numpy(sb.view(np.int32)).to(cuda)
    x = Q.synth_normal(oracle.activation_seed(70 + M), (M, K))

    # regular entry point on an uploaded handle
    qw = Q.QuantizedWeight.from_mlx(torch.from_numpy(w.view(np.int32)).view(torch.uint32),
                                    torch.from_numpy(s.view(np.int16)).view(torch.bfloat16),
                                    torch.from_numpy(b.view(np.int16)).view(torch.bfloat16))
    ref_logits = torch.empty((M, N), dtype=torch.bfloat16, device=cuda)
    rt, rv, rk = Q.lm_head_argmax(x, qw, softcap=30.0, rms_scale=True, row_offset=1000, logits=ref_logits)

    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    for call in range(2):      # two calls in a row share (and must clear) the static scratch
        logits = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device=cuda)
        tok = torch.full((M,), -1, dtype=torch.int32, device=cuda)
        val = torch.zeros((M,), dtype=torch.float32, device=cuda)
        key = torch.zeros((M,), dtype=torch.int64, device=cuda)
        _lib.call("g4q_lm_head_argmax_noalloc", _p(d_packed), _p(d_sb), N, K, _p(x), M, x.stride(0), 30.0,
                  _lib.QMM_RMS_SCALE, 1e-6, 1000, _p(logits), N, _p(tok), _p(val), _p(key), stream)
        torch.cuda.synchronize()
        assert torch.equal(tok, rt) and torch.equal(key, rk)
        assert torch.allclose(val, rv)
        # logits within the matmul tolerance of the regular entry point's (same kernel: identical)
        assert_qmm_close(oracle.bf16_to_f32(u16(logits)), oracle.bf16_to_f32(u16(ref_logits)).astype(np.float64),
                         bf16_out=True)
    assert _lib.device_error() == 0
    qw.free()


def test_noalloc_rejects_sizes_beyond_the_scratch(cuda):
    from helios_b200 import _lib
    from helios_b200 import quantized as Q
    x = torch.zeros((17, 64), dtype=torch.bfloat16, device=cuda)
    d = torch.zeros(1024, dtype=torch.int32, device=cuda)
    with pytest.raises(_lib.G4qInvalidArgument, match="static scratch holds 16 keys"):
        _lib.call("g4q_lm_head_argmax_noalloc", _p(d), _p(d), 64, 64, _p(x), 17, 64, 30.0, 0, 1e-6, 0, None, 0,
                  None, None, None, None)


def test_noalloc_reports_an_out_of_range_scale(cuda, oracle):
    """A caller-owned weight is never scanned at load time, so the kernel checks the scales it reads:
    one scale of 2^121 (beyond the fast dequantisation's |scale| < 2^120) records code 50 in the
    error word g4q_device_error reports; reading it with reset clears it, and a clean weight then
    leaves it at zero."""
    from helios_b200 import _lib
    from helios_b200 import quantized as Q
    N, K = 4096, 256
    w, s, b = oracle.synth_matrix(oracle.matrix_seed(3, 7), N, K)
    x = Q.synth_normal(oracle.activation_seed(90), (1, K))
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    tok = torch.empty((1,), dtype=torch.int32, device=cuda)

    def run(scales):
        packed, sb = oracle.repack(w, scales, b)
        d_packed = torch.from_numpy(packed.view(np.int32)).to(cuda)
        d_sb = torch.from_numpy(sb.view(np.int32)).to(cuda)
        _lib.call("g4q_lm_head_argmax_noalloc", _p(d_packed), _p(d_sb), N, K, _p(x), 1, K, 30.0, 0, 1e-6, 0, None,
                  0, _p(tok), None, None, stream)
        torch.cuda.synchronize()

    assert _lib.device_error() == 0
    bad = s.copy()
    bad[1234, 2] = 0x7C00            # bf16 2^121
    run(bad)
    assert _lib.device_error(reset=False) == 50
    assert _lib.device_error(reset=True) == 50
    assert _lib.device_error() == 0
    run(s)
    assert _lib.device_error() == 0
