"""MLX checkpoint loading for the quantized linears: the part of the reference's model load that the
kernels consume.

The reference reads `config.json` into a manifest (native/gemma4_mlx/src/model_manifest.cc:100-238:
default quantization bits/group_size, per-module overrides keyed by ``language_model.model.*`` and
limited to 4/8 bits at group 64, `:146-152`), loads every ``language_model.model.*`` tensor of the
safetensors shards into a name map (native_model.cc:84-104, NativeTextModel::load :3506-3590) and
looks up ``{prefix}.weight/.scales/.biases`` plus the spec of ``prefix`` at each call
(`quantization_for`, :208-215; `quantized_linear`, :349-362). Here the same names and specs feed
:class:`~helios_b200.quantized.QuantizedWeight` uploads (repacked on the device, tensor-parallel
windows taken at upload). Layer structure follows the reference graph: every sixth layer is a
full-attention layer (`target_layer_full_attention`, :494-496) with head_dim 512, one KV head and
no v_proj (k is reused as v, :813-822); the others have head_dim 256 and 8 KV heads.
"""
from __future__ import annotations

import json
import os
from dataclasses import dataclass, field
from pathlib import Path
from typing import Dict, Optional, Tuple

import torch

LANG = "language_model.model."
LINEARS = {"q": "self_attn.q_proj", "k": "self_attn.k_proj", "v": "self_attn.v_proj", "o": "self_attn.o_proj",
           "gate": "mlp.gate_proj", "up": "mlp.up_proj", "down": "mlp.down_proj"}
COLUMN_SPLIT = ("q", "k", "v", "gate", "up")   # output rows split across ranks
ROW_SPLIT = ("o", "down")                      # input columns split across ranks (group aligned)


class CheckpointError(ValueError):
    """The checkpoint does not match what the quantized linears need (the reference's load errors)."""


@dataclass
class Manifest:
    bits: int
    group_size: int
    overrides: Dict[str, Tuple[int, int]] = field(default_factory=dict)
    text: dict = field(default_factory=dict)
    tie_word_embeddings: bool = True
    attention_k_eq_v: bool = True

    def quantization_for(self, prefix: str) -> Tuple[int, int]:
        """(bits, group_size) of the module ``prefix``: its override, else the default."""
        return self.overrides.get(prefix, (self.bits, self.group_size))


def read_manifest(path, strict_12b: bool = False) -> Manifest:
    """Parse ``config.json`` of an MLX checkpoint directory (or the file itself)."""
    p = Path(path)
    cfg = json.loads((p / "config.json" if p.is_dir() else p).read_text())
    q = cfg.get("quantization_config", cfg.get("quantization"))
    if not isinstance(q, dict) or "bits" not in q or "group_size" not in q:
        raise CheckpointError("config.json is missing quantization bits/group_size")
    man = Manifest(bits=int(q["bits"]), group_size=int(q["group_size"]))
    for key, val in q.items():
        if not key.startswith(LANG) or not isinstance(val, dict) or "bits" not in val:
            continue
        spec = (int(val["bits"]), int(val.get("group_size", man.group_size)))
        if spec[1] != 64 or spec[0] not in (4, 8):
            raise CheckpointError(f"unsupported quantization override for {key}")
        man.overrides[key] = spec
    text = cfg.get("text_config", cfg)
    man.text = dict(text)
    man.tie_word_embeddings = bool(text.get("tie_word_embeddings", cfg.get("tie_word_embeddings", True)))
    man.attention_k_eq_v = bool(text.get("attention_k_eq_v", True))
    if strict_12b:
        want = dict(hidden_size=3840, intermediate_size=15360, num_hidden_layers=48, num_attention_heads=16,
                    num_key_value_heads=8, vocab_size=262144)
        bad = [k for k, v in want.items() if int(text.get(k, -1)) != v]
        if bad or (man.bits, man.group_size) != (4, 64) or not man.attention_k_eq_v or not man.tie_word_embeddings:
            raise CheckpointError(f"config.json does not match the Gemma 4 12B text shape ({', '.join(bad)})")
    return man


def full_attention(layer: int) -> bool:
    return (layer + 1) % 6 == 0


class Checkpoint:
    """The ``language_model.model.*`` tensors of an MLX checkpoint directory (lazily read)."""

    def __init__(self, path, strict_12b: bool = False):
        from safetensors import safe_open
        self.path = Path(path)
        self.manifest = read_manifest(self.path, strict_12b)
        files = sorted(f for f in os.listdir(self.path) if f.endswith(".safetensors"))
        if not files:
            raise CheckpointError(f"no .safetensors files in {self.path}")
        self._handles = [safe_open(str(self.path / f), framework="pt") for f in files]
        self._where: Dict[str, int] = {}
        self.total_tensors = 0
        for i, h in enumerate(self._handles):
            for name in h.keys():
                self.total_tensors += 1
                if name.startswith(LANG):
                    self._where[name] = i

    def names(self):
        return sorted(self._where)

    def has(self, name: str) -> bool:
        return name in self._where

    def tensor(self, name: str) -> torch.Tensor:
        if name not in self._where:
            raise CheckpointError(f"missing loaded tensor {name}")
        return self._handles[self._where[name]].get_tensor(name)

    def linear_arrays(self, prefix: str):
        """(weight uint32 [N, K*bits/32], scales bf16, biases bf16, bits, group_size) of ``prefix``."""
        bits, gs = self.manifest.quantization_for(prefix)
        w, s, b = (self.tensor(f"{prefix}.{n}") for n in ("weight", "scales", "biases"))
        if w.dtype not in (torch.uint32, torch.int32):
            raise CheckpointError(f"{prefix}.weight is {w.dtype}, expected packed uint32")
        K = w.shape[1] * 32 // bits
        if s.shape != (w.shape[0], K // gs) or b.shape != s.shape:
            raise CheckpointError(f"{prefix}: scales/biases shape {tuple(s.shape)} does not match {bits}-bit group {gs}")
        return w, s, b, bits, gs

    def linear(self, prefix: str, rows: Optional[Tuple[int, int]] = None, cols: Optional[Tuple[int, int]] = None):
        """Upload ``prefix`` (optionally a row / group-aligned column window) as a QuantizedWeight."""
        from .quantized import QuantizedWeight
        w, s, b, bits, gs = self.linear_arrays(prefix)
        return QuantizedWeight.from_mlx(w, s, b, bits=bits, group_size=gs, rows=rows, cols=cols)

    def layer_prefix(self, layer: int, name: str) -> str:
        return f"{LANG}layers.{layer}.{LINEARS[name]}"

    def layer_windows(self, layer: int, tp_rank: int = 0, tp_size: int = 1):
        """{name: (prefix, rows, cols)} of one layer's linears on rank ``tp_rank`` of ``tp_size``.
        Column-split rows for q/k/v/gate/up, group-aligned row split for o/down; a full-attention
        layer's single KV head (k, reused as v) is replicated on every rank."""
        out = {}
        for name in LINEARS:
            prefix = self.layer_prefix(layer, name)
            if name == "v" and full_attention(layer) and self.manifest.attention_k_eq_v:
                if self.has(prefix + ".weight"):
                    raise CheckpointError(f"{prefix} present on a full-attention layer with k_eq_v")
                continue
            w, s, b, bits, gs = self.linear_arrays(prefix)
            N, K = w.shape[0], w.shape[1] * 32 // bits
            rows = cols = None
            if tp_size > 1 and not (name == "k" and full_attention(layer)):
                if name in COLUMN_SPLIT:
                    if N % (tp_size * 16):
                        raise CheckpointError(f"{prefix}: {N} rows do not split into {tp_size} x 16-row shards")
                    n = N // tp_size
                    rows = (tp_rank * n, (tp_rank + 1) * n)
                else:
                    if K % (tp_size * gs):
                        raise CheckpointError(f"{prefix}: {K} columns do not split into {tp_size} group-aligned shards")
                    k = K // tp_size
                    cols = (tp_rank * k, (tp_rank + 1) * k)
            out[name] = (prefix, rows, cols)
        return out

    def load_layer(self, layer: int, tp_rank: int = 0, tp_size: int = 1):
        """{name: QuantizedWeight} of one layer (``v`` absent on full-attention layers: k is v)."""
        return {name: self.linear(prefix, rows, cols)
                for name, (prefix, rows, cols) in self.layer_windows(layer, tp_rank, tp_size).items()}

    def load_embed(self, tp_rank: int = 0, tp_size: int = 1):
        """The tied embedding / LM-head table; with ``tp_size`` > 1 the rank's vocabulary shard."""
        prefix = f"{LANG}embed_tokens"
        w = self.tensor(prefix + ".weight")
        rows = None
        if tp_size > 1:
            n = w.shape[0] // tp_size
            rows = (tp_rank * n, (tp_rank + 1) * n)
        return self.linear(prefix, rows=rows)
