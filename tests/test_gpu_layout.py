"""GPU: seeded generator, loader repack (host and device sources, windows, concatenation) and
bit-exact dequantize against the CPU oracle, through the C ABI."""
import json

import numpy as np
import pytest
import torch

from conftest import GOLDEN
from gpu_util import dev_u16, dev_u32, u16, u32

pytestmark = pytest.mark.gpu


def test_gpu_generator_matches_oracle(cuda, oracle):
    from helios_b200 import quantized as Q
    for seed, N, K in ((oracle.matrix_seed(0, 5), 256, 3840), (oracle.matrix_seed(47, 6), 48, 1024), (5, 16, 64)):
        w, s, b = Q.synth_matrix(seed, N, K)
        ow, os_, ob = oracle.synth_matrix(seed, N, K)
        assert (u32(w) == ow).all() and (u16(s) == os_).all() and (u16(b) == ob).all()
    x = Q.synth_normal(oracle.activation_seed(3), (7, 3840))
    assert (u16(x).ravel() == oracle.synth_normal_bf16(oracle.activation_seed(3), 7 * 3840)).all()
    w8, s8, b8 = Q.synth_matrix(77, 32, 256, bits=8)
    ow8, os8, ob8 = oracle.synth_matrix(77, 32, 256, bits=8)
    assert (u32(w8) == ow8).all() and (u16(s8) == os8).all()


@pytest.mark.parametrize("source", ["host", "device"])
def test_upload_export_roundtrip(cuda, oracle, source):
    from helios_b200.quantized import QuantizedWeight
    w, s, b = oracle.synth_matrix(oracle.matrix_seed(2, 3), 96, 640)
    if source == "host":
        tw = torch.from_numpy(w.view(np.int32)).view(torch.uint32)
        ts = torch.from_numpy(s.view(np.int16)).view(torch.bfloat16)
        tb = torch.from_numpy(b.view(np.int16)).view(torch.bfloat16)
    else:
        tw, ts, tb = dev_u32(w, cuda), dev_u16(s, cuda), dev_u16(b, cuda)
    q = QuantizedWeight.from_mlx(tw, ts, tb)
    assert q.info()["fast_path_ok"] == 1
    ew, es, eb = q.export()
    assert (u32(ew) == w).all() and (u16(es) == s).all() and (u16(eb) == b).all()
    q.free()


def test_layout_matches_oracle_repack(cuda, oracle):
    """The device layout equals the oracle's layout-v1 words (read back via a kernel-free path)."""
    from helios_b200 import quantized as Q
    z = np.load(GOLDEN / "small_matrix.npz")
    q = Q.QuantizedWeight.from_mlx(dev_u32(z["w"], cuda), dev_u16(z["scales"], cuda), dev_u16(z["biases"], cuda))
    d = Q.dequantize(q)
    assert (u16(d) == z["deq_r2"]).all()
    d1 = Q.dequantize(q, chain=Q.CHAIN_R1)
    assert (u16(d1) == z["deq_r1"]).all()


def test_windows_and_concat(cuda, oracle):
    from helios_b200.quantized import QuantizedWeight, dequantize
    w, s, b = oracle.synth_matrix(11, 128, 512)
    full = oracle.dequantize(w, s, b)
    tw, ts, tb = dev_u32(w, cuda), dev_u16(s, cuda), dev_u16(b, cuda)
    col = QuantizedWeight.from_mlx(tw, ts, tb, rows=(32, 96))
    assert (u16(dequantize(col)) == full[32:96]).all()
    row = QuantizedWeight.from_mlx(tw, ts, tb, cols=(128, 384))
    assert (u16(dequantize(row)) == full[:, 128:384]).all()
    w2, s2, b2 = oracle.synth_matrix(12, 64, 512)
    cat = QuantizedWeight.concat([(tw, ts, tb, (16, 48)), (dev_u32(w2, cuda), dev_u16(s2, cuda), dev_u16(b2, cuda))])
    ref = np.concatenate([full[16:48], oracle.dequantize(w2, s2, b2)])
    assert (u16(dequantize(cat)) == ref).all()


@pytest.mark.parametrize("chain", [1, 2])
def test_dequantize_full_size_bit_exact(cuda, oracle, chain):
    from helios_b200 import quantized as Q
    for proj, (N, K) in (("gate", (15360, 3840)), ("down", (3840, 15360)), ("o", (3840, 4096))):
        seed = oracle.matrix_seed(0, oracle.PROJ_IDS[proj])
        w, s, b = Q.synth_matrix(seed, N, K)
        q = Q.QuantizedWeight.from_mlx(w, s, b)
        d = u16(Q.dequantize(q, chain=chain))
        ow, os_, ob = oracle.synth_matrix(seed, N, K)
        ref = oracle.dequantize(ow, os_, ob, chain=chain)
        assert (d == ref).all(), f"{proj}: {(d != ref).sum()} mismatches"
        # the MLX-layout path agrees too
        d2 = u16(Q.dequantize(w, s, b, chain=chain))
        assert (d2 == ref).all()
        q.free()


def test_dequantize_special_values(cuda, oracle):
    """Every (scale, bias) of the known-answer file in one matrix: subnormals, signed zeros,
    huge exponent gaps, R1 != R2 cases; checked element by element against exact arithmetic."""
    from helios_b200 import quantized as Q
    kat = [c for c in json.loads((GOLDEN / "deq_kat.json").read_text())["cases"]
           if (c["r1"] >> 7) & 0xFF != 0xFF and (c["r2"] >> 7) & 0xFF != 0xFF]
    G = 64
    N = 16 * ((len(kat) + 16 * G - 1) // (16 * G))
    rng = np.random.default_rng(0)
    s = np.full((N, G), oracle.f32_to_bf16(np.float32(1.0)), dtype=np.uint16)
    b = np.zeros((N, G), dtype=np.uint16)
    for i, c in enumerate(kat):
        s[i // G, i % G] = c["scale"]
        b[i // G, i % G] = c["bias"]
    w = rng.integers(0, 2 ** 32, size=(N, G * 8), dtype=np.uint32)
    for chain in (1, 2):
        ref = oracle.dequantize(w, s, b, chain=chain)
        got = u16(Q.dequantize(dev_u32(w, cuda), dev_u16(s, cuda), dev_u16(b, cuda), chain=chain))
        nan = ((ref >> 7) & 0xFF == 0xFF) & ((ref & 0x7F) != 0)
        assert ((got == ref) | nan).all(), np.argwhere((got != ref) & ~nan)[:5]
        q = Q.QuantizedWeight.from_mlx(dev_u32(w, cuda), dev_u16(s, cuda), dev_u16(b, cuda))
        got2 = u16(Q.dequantize(q, chain=chain))
        assert ((got2 == ref) | nan).all()
        q.free()


def test_dequantize_rows_gather(cuda, oracle):
    from helios_b200 import quantized as Q
    seed = oracle.matrix_seed(0, 7)
    w, s, b = Q.synth_matrix(seed, 4096, 3840)
    q = Q.QuantizedWeight.from_mlx(w, s, b)
    ids = torch.tensor([0, 4095, 17, 17, 2048, 9], dtype=torch.int32, device=cuda)
    got = u16(Q.dequantize(q, rows=ids))
    ow, os_, ob = oracle.synth_matrix(seed, 4096, 3840)
    ref = oracle.dequantize_rows(ow, os_, ob, ids.cpu().numpy())
    assert (got == ref).all()
    assert q.info()["error_flags"] == 0
    bad = Q.dequantize(q, rows=torch.tensor([1, 4096], dtype=torch.int32, device=cuda))
    assert (u16(bad[1]) == 0).all() and q.info()["error_flags"] & 2
    q.free()


@pytest.mark.parametrize("bits,gs", [(4, 32), (4, 128), (8, 64), (8, 32)])
def test_dequantize_mlx_other_formats(cuda, oracle, bits, gs):
    from helios_b200 import quantized as Q
    w, s, b = Q.synth_matrix(1234 + bits + gs, 64, 512, bits=bits, group_size=gs)
    ow, os_, ob = oracle.synth_matrix(1234 + bits + gs, 64, 512, bits=bits, group_size=gs)
    for chain in (1, 2):
        ref = oracle.dequantize(ow, os_, ob, bits=bits, group_size=gs, chain=chain)
        got = u16(Q.dequantize(w, s, b, group_size=gs, bits=bits, chain=chain))
        assert (got == ref).all()
