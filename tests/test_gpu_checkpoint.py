"""GPU: a small synthetic MLX checkpoint loaded through the checkpoint loader into libg4q weights
(repacked on the device, tensor-parallel windows, the 8-bit override on the generic path, the
full-attention layer without v_proj); every uploaded matrix dequantizes bit-exactly to the oracle's
dequantize of the same window."""
import pytest

import ckpt_util
from gpu_util import u16

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("tp_rank,tp_size", [(0, 1), (1, 2)])
def test_checkpoint_layers_upload_bit_exact(cuda, oracle, tmp_path, tp_rank, tp_size):
    from helios_b200 import checkpoint as C
    from helios_b200 import quantized as Q
    arrays = ckpt_util.write(tmp_path, oracle)
    ck = C.Checkpoint(tmp_path)
    for layer in (0, 5):
        wins = ck.layer_windows(layer, tp_rank, tp_size)
        ws = ck.load_layer(layer, tp_rank, tp_size)
        assert set(ws) == set(wins)
        for name, q in ws.items():
            prefix, rows, cols = wins[name]
            w, s, b, bits = arrays[prefix]
            full = oracle.dequantize(w, s, b, bits=bits, group_size=64)
            r0, r1 = rows or (0, full.shape[0])
            c0, c1 = cols or (0, full.shape[1])
            assert q.bits == bits and q.shape == (r1 - r0, c1 - c0)
            assert (u16(Q.dequantize(q, bits=bits, group_size=64)) == full[r0:r1, c0:c1]).all(), prefix
            q.free()
    emb = ck.load_embed(tp_rank, tp_size)
    w, s, b, _ = arrays["language_model.model.embed_tokens"]
    n = w.shape[0] // tp_size
    assert (u16(Q.dequantize(emb)) == oracle.dequantize(w, s, b)[tp_rank * n:(tp_rank + 1) * n]).all()
    emb.free()
