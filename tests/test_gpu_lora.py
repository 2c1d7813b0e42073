"""GPU: the LoRA delta on a quantized linear's output (add_lora_delta_if_active,
native/gemma4_mlx/src/native_model.cc:316-328) against the CPU oracle, through the C ABI.

The oracle accumulates both low-rank products in float64 and rounds each once to fp32; the kernels
accumulate in fp32 in another order, so the bf16 results may differ by one ulp where the fp32 delta
lies next to a bf16 rounding boundary. Checked: at least 99% of the outputs bit-identical and
max|y - y_oracle| <= 1e-2 * rms(y_oracle) (the north star's matmul tolerance)."""
import ctypes

import numpy as np
import pytest
import torch

from gpu_util import dev_u16, u16

pytestmark = pytest.mark.gpu


def lora_mats(rank, K, N, seed):
    g = torch.Generator().manual_seed(seed)
    a = torch.randn(rank, K, generator=g) / K ** 0.5
    b = torch.randn(N, rank, generator=g) / rank ** 0.5
    return a, b


def check(oracle, y_gpu_bits, y_ref_bits):
    yg = oracle.bf16_to_f32(y_gpu_bits).astype(np.float64)
    yr = oracle.bf16_to_f32(y_ref_bits).astype(np.float64)
    rms = float(np.sqrt(np.mean(yr ** 2)))
    assert np.abs(yg - yr).max() <= 1e-2 * rms, (np.abs(yg - yr).max(), rms)
    assert (y_gpu_bits == y_ref_bits).mean() >= 0.99, (y_gpu_bits == y_ref_bits).mean()


@pytest.mark.parametrize("M", [1, 2, 8])
def test_lora_delta_decode_widths_q_proj(cuda, oracle, M):
    from helios_b200 import quantized as Q
    N, K, rank, alpha = 4096, 3840, 16, 32.0
    seed = oracle.matrix_seed(0, oracle.PROJ_IDS["q"])
    w, s, b = Q.synth_matrix(seed, N, K)
    qw = Q.QuantizedWeight.from_mlx(w, s, b)
    x = Q.synth_normal(oracle.activation_seed(M), (M, K))
    a, bm = lora_mats(rank, K, N, M)
    lora = Q.LoraAdapter(a, bm, alpha, max_tokens=8)
    base = Q.quantized_matmul(x, qw)
    y = Q.quantized_linear(x, qw, lora)
    torch.cuda.synchronize()
    ref = oracle.lora_delta(u16(x), u16(base), a.numpy(), bm.numpy(), alpha)
    check(oracle, u16(y), ref)
    # the delta is not negligible next to the base output
    assert (u16(y) != u16(base)).mean() > 0.9
    lora.free()
    qw.free()


def test_lora_delta_ragged_strided_chunked(cuda, oracle):
    """rank 5 (a partial warp group), N = 1000 (a partial CTA), K = 136, M = 37 in chunks of 16
    tokens, row strides wider than the rows, host-memory A and B."""
    from helios_b200 import _lib
    from helios_b200 import quantized as Q
    M, N, K, rank, alpha = 37, 1000, 136, 5, 7.0
    ldx, ldy = 144, 1016
    a, bm = lora_mats(rank, K, N, 11)
    g = torch.Generator().manual_seed(12)
    xs = torch.randn(M, ldx, generator=g).to(torch.bfloat16).to(cuda)
    ys = torch.randn(M, ldy, generator=g).to(torch.bfloat16).to(cuda)
    y0 = u16(ys).copy()
    lora = Q.LoraAdapter(a, bm, alpha, max_tokens=16)
    _lib.call("g4q_lora_apply", lora.handle, ctypes.c_void_p(xs.data_ptr()), M, ldx,
              ctypes.c_void_p(ys.data_ptr()), ldy, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    yg = u16(ys)
    ref = oracle.lora_delta(u16(xs)[:, :K], y0[:, :N], a.numpy(), bm.numpy(), alpha)
    check(oracle, yg[:, :N], ref)
    assert (yg[:, N:] == y0[:, N:]).all()      # the padding columns are not touched
    lora.free()


def test_lora_delta_prefill_down_proj(cuda, oracle):
    """M = 300 tokens through the prefill GEMM's output shape (down_proj 3840 x 15360), rank 64,
    device-memory A and B in bf16 (converted to fp32 as the reference does)."""
    from helios_b200 import quantized as Q
    M, N, K, rank, alpha = 300, 3840, 15360, 64, 16.0
    a, bm = lora_mats(rank, K, N, 3)
    a16, b16 = a.to(torch.bfloat16), bm.to(torch.bfloat16)
    x = Q.synth_normal(oracle.activation_seed(5), (M, K))
    g = torch.Generator().manual_seed(4)
    y = (3.0 * torch.randn(M, N, generator=g)).to(torch.bfloat16).to(cuda)
    y0 = u16(y).copy()
    lora = Q.LoraAdapter(a16.to(cuda), b16.to(cuda), alpha, max_tokens=128)
    lora.apply(x, y)
    torch.cuda.synchronize()
    ref = oracle.lora_delta(u16(x), y0, a16.float().numpy(), b16.float().numpy(), alpha)
    check(oracle, u16(y), ref)
    lora.free()


def test_lora_apply_replays_in_a_cuda_graph(cuda, oracle):
    """apply allocates nothing (the low-rank scratch belongs to the handle), so it can be captured."""
    from helios_b200 import quantized as Q
    M, N, K, rank, alpha = 2, 2048, 3840, 8, 16.0
    a, bm = lora_mats(rank, K, N, 21)
    lora = Q.LoraAdapter(a, bm, alpha, max_tokens=2)
    x = Q.synth_normal(oracle.activation_seed(9), (M, K))
    base = dev_u16(np.zeros((M, N), np.uint16), cuda)
    y = torch.empty_like(base)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        y.copy_(base)
        lora.apply(x, y)                      # warm-up outside the capture
    torch.cuda.current_stream().wait_stream(s)
    eager = u16(y).copy()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        y.copy_(base)
        lora.apply(x, y)
    y.fill_(1.0)
    graph.replay()
    torch.cuda.synchronize()
    assert (u16(y) == eager).all()
    ref = oracle.lora_delta(u16(x), u16(base), a.numpy(), bm.numpy(), alpha)
    check(oracle, eager, ref)
    del graph
    lora.free()
