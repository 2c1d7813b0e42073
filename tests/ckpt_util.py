"""A small synthetic MLX checkpoint (config.json + one safetensors shard) for the loader tests:
6 layers so that layer 5 is a full-attention layer (head_dim x 2, one KV head, no v_proj), one
8-bit per-module override, and a tensor outside language_model.model.* that the loader skips."""
import json

import numpy as np
import torch

HIDDEN, INTER, VOCAB = 128, 256, 512
SLIDE = dict(q=256, k=128, v=128)   # rows of the sliding layers' q/k/v
FULL = dict(q=512, k=64)            # full-attention layer: no v
OVERRIDE = "language_model.model.layers.0.mlp.down_proj"


def shapes(layer):
    full = (layer + 1) % 6 == 0
    qkv = FULL if full else SLIDE
    out = {f"self_attn.{n}_proj": (r, HIDDEN) for n, r in qkv.items()}
    out["self_attn.o_proj"] = (HIDDEN, qkv["q"])
    out["mlp.gate_proj"] = (INTER, HIDDEN)
    out["mlp.up_proj"] = (INTER, HIDDEN)
    out["mlp.down_proj"] = (HIDDEN, INTER)
    return out


def write(path, oracle, override_group=64):
    """Write the checkpoint; returns {prefix: (w, s, b, bits)} as numpy arrays."""
    from safetensors.torch import save_file
    tensors, arrays = {}, {}
    mats = {f"language_model.model.layers.{i}.{n}": rc for i in range(6) for n, rc in shapes(i).items()}
    mats["language_model.model.embed_tokens"] = (VOCAB, HIDDEN)
    for j, (prefix, (N, K)) in enumerate(sorted(mats.items())):
        bits = 8 if prefix == OVERRIDE else 4
        w, s, b = oracle.synth_matrix(900 + j, N, K, bits=bits, group_size=64)
        arrays[prefix] = (w, s, b, bits)
        tensors[prefix + ".weight"] = torch.from_numpy(w.view(np.int32)).view(torch.uint32)
        tensors[prefix + ".scales"] = torch.from_numpy(s.view(np.int16)).view(torch.bfloat16)
        tensors[prefix + ".biases"] = torch.from_numpy(b.view(np.int16)).view(torch.bfloat16)
    tensors["vision_tower.patch_embed.weight"] = torch.zeros(4, 4)
    save_file(tensors, str(path / "model.safetensors"))
    cfg = {"architectures": ["Gemma4UnifiedForConditionalGeneration"], "model_type": "gemma4_unified",
           "quantization": {"bits": 4, "group_size": 64, OVERRIDE: {"bits": 8, "group_size": override_group}},
           "text_config": {"hidden_size": HIDDEN, "intermediate_size": INTER, "num_hidden_layers": 6,
                           "num_attention_heads": 2, "num_key_value_heads": 1, "vocab_size": VOCAB,
                           "attention_k_eq_v": True, "tie_word_embeddings": True}}
    (path / "config.json").write_text(json.dumps(cfg))
    return arrays
