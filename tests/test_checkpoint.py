"""CPU: the MLX checkpoint loader's manifest, names, specs and tensor-parallel windows, on a small
synthetic checkpoint (the quantized-linear part of the reference's model load)."""
import json

import numpy as np
import pytest

import ckpt_util


def test_manifest_and_specs(tmp_path, oracle):
    from helios_b200 import checkpoint as C
    ckpt_util.write(tmp_path, oracle)
    man = C.read_manifest(tmp_path)
    assert (man.bits, man.group_size) == (4, 64)
    assert man.quantization_for(ckpt_util.OVERRIDE) == (8, 64)
    assert man.quantization_for("language_model.model.layers.1.mlp.down_proj") == (4, 64)
    with pytest.raises(C.CheckpointError):
        C.read_manifest(tmp_path, strict_12b=True)   # not the 12B shape


def test_override_limits(tmp_path, oracle):
    """Overrides other than 4/8 bits at group 64 are rejected, as the reference's manifest does."""
    from helios_b200 import checkpoint as C
    ckpt_util.write(tmp_path, oracle, override_group=32)
    with pytest.raises(C.CheckpointError):
        C.read_manifest(tmp_path)
    cfg = json.loads((tmp_path / "config.json").read_text())
    del cfg["quantization"]
    (tmp_path / "config.json").write_text(json.dumps(cfg))
    with pytest.raises(C.CheckpointError):
        C.read_manifest(tmp_path)


def test_names_arrays_and_windows(tmp_path, oracle):
    from helios_b200 import checkpoint as C
    arrays = ckpt_util.write(tmp_path, oracle)
    ck = C.Checkpoint(tmp_path)
    assert all(n.startswith(C.LANG) for n in ck.names())
    assert ck.total_tensors == len(ck.names()) + 1        # the vision tensor is seen, not kept
    w, s, b, bits, gs = ck.linear_arrays(ckpt_util.OVERRIDE)
    ow, os_, ob, obits = arrays[ckpt_util.OVERRIDE]
    assert (bits, gs) == (8, 64) and (w.numpy().view(np.uint32) == ow).all()
    # sliding layer, 2 ranks: column split rows, row split columns
    win = ck.layer_windows(0, tp_rank=1, tp_size=2)
    assert set(win) == {"q", "k", "v", "o", "gate", "up", "down"}
    assert win["q"][1] == (128, 256) and win["k"][1] == (64, 128) and win["gate"][1] == (128, 256)
    assert win["o"][2] == (128, 256) and win["down"][2] == (128, 256) and win["o"][1] is None
    # full-attention layer: no v (k is v), the single KV head is replicated
    full = ck.layer_windows(5, tp_rank=1, tp_size=2)
    assert "v" not in full and full["k"][1] is None and full["q"][1] == (256, 512)
    with pytest.raises(C.CheckpointError):
        ck.tensor("language_model.model.layers.9.mlp.up_proj.weight")
