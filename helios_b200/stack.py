"""Synthetic Gemma-style decoder stack built from the quantized linears only.

This is the workload of the benchmark configs (48 layers of the seven 4-bit g64 projections
plus the quantized tied LM head). It stands in for the linear part of the reference's decode
and prefill drivers (native_model.cc:1843-1911 ``decode_last_logits``, :1682-1780
``decode_block_hidden``/``forward_hidden``, :1819-1841 chunked prefill): the same 336 + 1
quantized matmuls per step in the same order, with attention, RoPE, GeGLU and the KV cache left
out (outside the quantized-linear path). Data flow per layer, with ``rms(v)`` the RMSNorm scale
``1/sqrt(mean(v^2)+eps)`` folded into the consuming matmul's epilogue:

    qkv = rms(h) * (h @ [Wq|Wk|Wv]^T)        # q|k|v share their input: one fused launch
    o   = q @ Wo^T                           # q stands in for the attention output
    gu  = rms(o) * (o @ [Wgate|Wup]^T)       # gate|up share their input: one fused launch
    h   = up @ Wdown^T                       # up stands in for the GeGLU output
    logits = rms(h) * (h @ Wlm^T); token = argmax(softcap(logits))

Tensor parallelism over ``tp_size`` GPUs (one process each): q/k/v/gate/up/LM-head rows are
split (column-parallel), o/down columns are split along K at group boundaries (row-parallel),
o/down emit fp32 partial sums that are summed across ranks (allreduce) and rounded to bf16,
and the LM-head shards combine their 64-bit argmax keys with a max.
"""
from __future__ import annotations

import struct
from dataclasses import dataclass
from typing import List, Optional

import torch

from .quantized import (PHASE_ALLREDUCE, PHASE_ARGMAX, PHASE_GEGLU, QMM_RMS_SCALE, DecodePlan, QuantizedWeight,
                        lm_head_argmax, quantized_matmul, synth_matrix, synth_normal)

BASE_SEED = 0x48454C494F53
PROJ_IDS = {"q": 0, "k": 1, "v": 2, "o": 3, "gate": 4, "up": 5, "down": 6, "lm": 7}


def matrix_seed(layer: int, proj: str) -> int:
    return BASE_SEED ^ ((0 if proj == "lm" else layer) * 16 + PROJ_IDS[proj])


def activation_seed(chunk: int) -> int:
    return BASE_SEED ^ 0xF00 ^ chunk


@dataclass
class StackConfig:
    layers: int = 48
    hidden: int = 3840
    q_out: int = 4096       # 16 heads x 256
    kv_out: int = 2048      # 8 KV heads x 256
    inter: int = 15360
    vocab: int = 262144
    softcap: float = 30.0
    eps: float = 1e-6

    def shapes(self):
        return {"q": (self.q_out, self.hidden), "k": (self.kv_out, self.hidden), "v": (self.kv_out, self.hidden),
                "o": (self.hidden, self.q_out), "gate": (self.inter, self.hidden), "up": (self.inter, self.hidden),
                "down": (self.hidden, self.inter), "lm": (self.vocab, self.hidden)}

    def weight_bytes(self) -> int:
        """Packed + scale/bias bytes of every matrix (0.5625 B per weight)."""
        sh = self.shapes()
        per_layer = sum(n * k for p, (n, k) in sh.items() if p != "lm")
        return int((per_layer * self.layers + sh["lm"][0] * sh["lm"][1]) * 9 // 16)

    def flops_per_token(self) -> int:
        sh = self.shapes()
        per_layer = sum(n * k for p, (n, k) in sh.items() if p != "lm")
        return 2 * per_layer * self.layers


def _split(n: int, rank: int, size: int, align: int) -> tuple:
    if n % (size * align) != 0:
        raise ValueError(f"dimension {n} does not split into {size} shards of multiples of {align}")
    step = n // size
    return rank * step, (rank + 1) * step


def shard_plan(cfg: "StackConfig", rank: int, size: int) -> dict:
    """Tensor-parallel windows of rank ``rank`` of ``size``: row windows (column-parallel q/k/v,
    gate/up, LM head; whole 16-row tiles) and K windows (row-parallel o, down; whole 64-groups)."""
    return {"q_rows": _split(cfg.q_out, rank, size, 16), "kv_rows": _split(cfg.kv_out, rank, size, 16),
            "i_rows": _split(cfg.inter, rank, size, 16), "v_rows": _split(cfg.vocab, rank, size, 16),
            "o_cols": _split(cfg.q_out, rank, size, 64), "d_cols": _split(cfg.inter, rank, size, 64)}


_SIGN = -(2 ** 63)


def combine_keys(keys: torch.Tensor, group=None) -> torch.Tensor:
    """Max over ranks of the 64-bit argmax keys (unsigned order): flip the top bit so a signed int64
    max orders them, all-reduce with MAX, flip back. Ties keep the smallest vocabulary index."""
    k = keys ^ _SIGN
    torch.distributed.all_reduce(k, op=torch.distributed.ReduceOp.MAX, group=group)
    return k ^ _SIGN


class SyntheticStack:
    """Seeded random-init weights of the synthetic stack, sharded for rank ``tp_rank`` of ``tp_size``."""

    def __init__(self, cfg: StackConfig, tp_rank: int = 0, tp_size: int = 1, group=None,
                 max_tokens: int = 16):
        self.cfg, self.rank, self.size, self.group = cfg, tp_rank, tp_size, group
        self.device = torch.device("cuda", torch.cuda.current_device())
        sh = cfg.shapes()
        plan = shard_plan(cfg, tp_rank, tp_size)
        self.q_rows, self.kv_rows, self.i_rows = plan["q_rows"], plan["kv_rows"], plan["i_rows"]
        self.o_cols, self.d_cols, self.v_rows = plan["o_cols"], plan["d_cols"], plan["v_rows"]
        self.nq = self.q_rows[1] - self.q_rows[0]
        self.nkv = self.kv_rows[1] - self.kv_rows[0]
        self.ni = self.i_rows[1] - self.i_rows[0]
        self.layers: List[dict] = []
        for layer in range(cfg.layers):
            mats = {p: synth_matrix(matrix_seed(layer, p), *sh[p]) for p in ("q", "k", "v")}
            qkv = QuantizedWeight.concat([(*mats["q"], self.q_rows), (*mats["k"], self.kv_rows),
                                          (*mats["v"], self.kv_rows)])
            del mats
            o = QuantizedWeight.from_mlx(*synth_matrix(matrix_seed(layer, "o"), *sh["o"]), cols=self.o_cols)
            mats = {p: synth_matrix(matrix_seed(layer, p), *sh[p]) for p in ("gate", "up")}
            gu = QuantizedWeight.concat([(*mats["gate"], self.i_rows), (*mats["up"], self.i_rows)])
            del mats
            down = QuantizedWeight.from_mlx(*synth_matrix(matrix_seed(layer, "down"), *sh["down"]), cols=self.d_cols)
            self.layers.append({"qkv": qkv, "o": o, "gu": gu, "down": down})
        self.lm = QuantizedWeight.from_mlx(*synth_matrix(matrix_seed(0, "lm"), *sh["lm"]), rows=self.v_rows)
        torch.cuda.synchronize()
        self._alloc(max_tokens)

    def _alloc(self, M: int):
        if getattr(self, "plan", None) is not None:
            raise RuntimeError("activation buffers are baked into the decode plan; build the stack with max_tokens >= M")
        dev, c = self.device, self.cfg
        self.max_tokens = M
        self.qkv_out = torch.empty((M, self.nq + 2 * self.nkv), dtype=torch.bfloat16, device=dev)
        self.o_out = torch.empty((M, c.hidden), dtype=torch.bfloat16, device=dev)
        self.gu_out = torch.empty((M, 2 * self.ni), dtype=torch.bfloat16, device=dev)
        self.h_out = torch.empty((M, c.hidden), dtype=torch.bfloat16, device=dev)
        self.part = torch.empty((M, c.hidden), dtype=torch.float32, device=dev)
        self.tokens = torch.empty(M, dtype=torch.int32, device=dev)
        self.values = torch.empty(M, dtype=torch.float32, device=dev)
        self.keys = torch.empty(M, dtype=torch.int64, device=dev)

    def _row_parallel(self, w: QuantizedWeight, x: torch.Tensor, out: torch.Tensor, part=None) -> torch.Tensor:
        """Row-parallel linear + the allreduce after it (fp32 partial sums, then one bf16 rounding)."""
        if self.size == 1:
            return quantized_matmul(x, w, out=out)
        part = self.part if part is None else part
        M = x.shape[0]
        quantized_matmul(x, w, out_dtype=torch.float32, out=part[:M])
        return self.sum_partials(part[:M], out)

    def sum_partials(self, p: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
        """The collective of a row-parallel linear: out (bf16) = sum over ranks of p (fp32 [M, cols]),
        as an NCCL allreduce of the fp32 partials and a cast. (A reduce-scatter of the fp32 partials
        followed by an all-gather of bf16 rows moves 3/4 of the bytes but measured slower at 2 GPUs for
        2048 x 3840 partials: 114 vs 89 us per sum, two collectives' latency instead of one.)"""
        torch.distributed.all_reduce(p, group=self.group)
        out.copy_(p)
        return out

    def forward(self, h: torch.Tensor):
        """One decode step (M <= max_tokens rows) or one prefill chunk; returns (tokens, values, h)."""
        M = h.shape[0]
        if M > self.max_tokens:
            self._alloc(M)
        c = self.cfg
        x = h
        for L in self.layers:
            qkv = quantized_matmul(x, L["qkv"], rms_scale=True, eps=c.eps, out=self.qkv_out[:M])
            o = self._row_parallel(L["o"], qkv[:, : self.nq], self.o_out[:M])
            gu = quantized_matmul(o, L["gu"], rms_scale=True, eps=c.eps, out=self.gu_out[:M])
            x = self._row_parallel(L["down"], gu[:, self.ni:], self.h_out[:M])
        return self.head(x)

    def prefill(self, h: torch.Tensor, sub_chunks: int = 1, head: bool = True):
        """One chunked-prefill chunk: M tokens through every layer's quantized
        linears on the tcgen05 GEMM (M > 16), then the LM head on the chunk's last row only.
        Uses its own activation buffers (the decode buffers stay baked into the plan).

        Tensor parallel, ``sub_chunks`` > 1: the chunk is cut into row blocks and the NCCL allreduce
        of one block's o/down partials runs on a second stream while the GEMMs of the next block
        run (the rows are independent; results are bit-identical to ``sub_chunks`` = 1). Measured
        on B200 at 2 GPUs it is slower (41.3 vs 33.8 ms per 2048-token chunk): the GEMM keeps one
        CTA on every SM, so the NCCL kernels wait for SMs instead of overlapping, and the half-height
        GEMMs lose tile efficiency. Off by default. ``head`` False skips the LM head (the chunks
        before the last one of a long prompt, as prefill_chunked_last_logits computes logits for the
        final chunk only). Returns (key of the last row or None, h)."""
        M = h.shape[0]
        c, dev = self.cfg, self.device
        pb = getattr(self, "_pre", None)
        if pb is None or pb["M"] < M:
            pb = {"M": M,
                  "qkv": torch.empty((M, self.nq + 2 * self.nkv), dtype=torch.bfloat16, device=dev),
                  "o": torch.empty((M, c.hidden), dtype=torch.bfloat16, device=dev),
                  "gu": torch.empty((M, 2 * self.ni), dtype=torch.bfloat16, device=dev),
                  "h": torch.empty((M, c.hidden), dtype=torch.bfloat16, device=dev),
                  "part": torch.empty((M, c.hidden), dtype=torch.float32, device=dev),
                  "part2": torch.empty((M, c.hidden), dtype=torch.float32, device=dev)}
            self._pre = pb
        if self.size == 1 or sub_chunks <= 1 or M < 2 * 256:
            x = h
            for L in self.layers:
                qkv = quantized_matmul(x, L["qkv"], rms_scale=True, eps=c.eps, out=pb["qkv"][:M])
                o = self._row_parallel(L["o"], qkv[:, : self.nq], pb["o"][:M], part=pb["part"])
                gu = quantized_matmul(o, L["gu"], rms_scale=True, eps=c.eps, out=pb["gu"][:M])
                x = self._row_parallel(L["down"], gu[:, self.ni:], pb["h"][:M], part=pb["part"])
            key = self.head(x[M - 1:M])[0] if head else None
            return key, x
        # row blocks on 256-row boundaries (the GEMM's token tile)
        step = -(-M // sub_chunks)
        step = -(-step // 256) * 256
        blocks = [(r0, min(M, r0 + step)) for r0 in range(0, M, step)]
        comp = torch.cuda.current_stream()
        comm = getattr(self, "_comm_stream", None)
        if comm is None:
            comm = self._comm_stream = torch.cuda.Stream(device=dev)
        comm.wait_stream(comp)

        def allreduce_async(part, out):
            ev = torch.cuda.Event()
            ev.record(comp)
            comm.wait_event(ev)
            with torch.cuda.stream(comm):
                torch.distributed.all_reduce(part, group=self.group)
                out.copy_(part)
            done = torch.cuda.Event()
            done.record(comm)
            return done

        x = h
        h_ready = [None] * len(blocks)   # event: block's input of this layer is ready
        for L in self.layers:
            o_ready = []
            for i, (r0, r1) in enumerate(blocks):
                if h_ready[i] is not None:
                    comp.wait_event(h_ready[i])
                qkv = quantized_matmul(x[r0:r1], L["qkv"], rms_scale=True, eps=c.eps, out=pb["qkv"][r0:r1])
                quantized_matmul(qkv[:, : self.nq], L["o"], out_dtype=torch.float32, out=pb["part"][r0:r1])
                o_ready.append(allreduce_async(pb["part"][r0:r1], pb["o"][r0:r1]))
            for i, (r0, r1) in enumerate(blocks):
                comp.wait_event(o_ready[i])
                gu = quantized_matmul(pb["o"][r0:r1], L["gu"], rms_scale=True, eps=c.eps, out=pb["gu"][r0:r1])
                quantized_matmul(gu[:, self.ni:], L["down"], out_dtype=torch.float32, out=pb["part2"][r0:r1])
                h_ready[i] = allreduce_async(pb["part2"][r0:r1], pb["h"][r0:r1])
            x = pb["h"]
        for ev in h_ready:
            comp.wait_event(ev)
        x = pb["h"][:M]
        key = self.head(x[M - 1:M])[0] if head else None
        return key, x

    def prefill_flops(self, M: int) -> int:
        """Whole-job FLOPs of one prefill chunk of M tokens (all ranks; LM head on one row)."""
        return self.cfg.flops_per_token() * M + 2 * self.cfg.vocab * self.cfg.hidden

    def build_plan(self, max_tokens: int = 1, keep_layers: bool = False) -> DecodePlan:
        """The whole decode step (48 x 4 matmuls + LM head argmax) as one persistent-kernel plan.

        Tensor parallel (``tp_size`` > 1, collective over the group): o and down are ALLREDUCE phases,
        their partial sums cross NVLink inside the kernel, and the LM-head keys are combined there too,
        so one step is one launch per GPU with no NCCL call.

        ``keep_layers``: every layer writes its own output buffers (``self.layer_outs[l]`` with
        ``qkv``, ``o``, ``gu``, ``h``) instead of reusing one set, so each phase's input and output
        stay readable after the step (the per-phase parity check). The kernel's work and dataflow
        are the same: each phase still reads the previous phase's output."""
        c = self.cfg
        if getattr(self, "plan", None) is not None:
            self.plan.free()
        self.h_in = torch.zeros((max(max_tokens, 1), c.hidden), dtype=torch.bfloat16, device=self.device)
        ar = PHASE_ALLREDUCE if self.size > 1 else 0
        phases, x = [], self.h_in
        self.layer_outs = []
        for L in self.layers:
            if keep_layers:
                M, dev = self.max_tokens, self.device
                bufs = {"qkv": torch.empty((M, self.nq + 2 * self.nkv), dtype=torch.bfloat16, device=dev),
                        "o": torch.empty((M, c.hidden), dtype=torch.bfloat16, device=dev),
                        "gu": torch.empty((M, 2 * self.ni), dtype=torch.bfloat16, device=dev),
                        "h": torch.empty((M, c.hidden), dtype=torch.bfloat16, device=dev)}
                self.layer_outs.append(bufs)
            else:
                bufs = {"qkv": self.qkv_out, "o": self.o_out, "gu": self.gu_out, "h": self.h_out}
            phases.append((L["qkv"], x, bufs["qkv"], QMM_RMS_SCALE))
            phases.append((L["o"], bufs["qkv"][:, : self.nq], bufs["o"], ar))
            phases.append((L["gu"], bufs["o"], bufs["gu"], QMM_RMS_SCALE))
            phases.append((L["down"], bufs["gu"][:, self.ni:], bufs["h"], ar))
            x = bufs["h"]
        self.h_last = x
        phases.append((self.lm, x, None, QMM_RMS_SCALE | PHASE_ARGMAX))
        self.plan = DecodePlan(phases, max_tokens, rank=self.rank, n_ranks=self.size, group=self.group)
        return self.plan

    def decode(self, h: torch.Tensor, logits: Optional[torch.Tensor] = None):
        """One decode step through the single-launch plan: h [M, hidden] -> (keys, final hidden).
        ``logits`` (bf16 [M, vocab shard]) also receives the LM head's pre-softcap logits."""
        M = h.shape[0]
        self.h_in[:M].copy_(h)
        self.plan.run(M, eps=self.cfg.eps, softcap=self.cfg.softcap, row_offset=self.v_rows[0],
                      tokens=self.tokens[:M], values=self.values[:M], keys=self.keys[:M], logits=logits)
        return self.keys[:M], self.h_last[:M]

    def gather_layer_outputs(self, M: int = 1, logits: Optional[torch.Tensor] = None):
        """The per-layer outputs of the last step of a ``keep_layers`` plan at full width, as bf16 bit
        patterns (numpy uint16) on rank 0: a list of dicts qkv (q|k|v), o, gu (gate|up), h, and the
        logits when given (the rank's vocabulary shard [M, rows]). Column-parallel shards are
        gathered over the group (a collective: every rank calls it); other ranks get None."""
        def bits(t):
            return t.contiguous().view(torch.int16).cpu().numpy().view("uint16")

        def gather(t):
            if self.size == 1:
                return [t]
            parts = [torch.empty_like(t) for _ in range(self.size)]
            torch.distributed.all_gather(parts, t.contiguous(), group=self.group)
            return parts

        outs = []
        for bufs in self.layer_outs:
            qkv = gather(bufs["qkv"][:M])
            gu = gather(bufs["gu"][:M])
            if self.rank == 0:
                q = [p[:, : self.nq] for p in qkv]
                k = [p[:, self.nq: self.nq + self.nkv] for p in qkv]
                v = [p[:, self.nq + self.nkv:] for p in qkv]
                g = [p[:, : self.ni] for p in gu]
                u = [p[:, self.ni:] for p in gu]
                outs.append({"qkv": bits(torch.cat(q + k + v, dim=1)), "o": bits(bufs["o"][:M]),
                             "gu": bits(torch.cat(g + u, dim=1)), "h": bits(bufs["h"][:M])})
        full_logits = None
        if logits is not None:
            lg = gather(logits[:M])
            if self.rank == 0:
                full_logits = bits(torch.cat(lg, dim=1))
        return (outs, full_logits) if self.rank == 0 else (None, None)

    def local_weight_bytes(self) -> int:
        """Packed + scale/bias bytes of this rank's shards (0.5625 B per weight)."""
        mats = [w for L in self.layers for w in L.values()] + [self.lm]
        return sum(w.rows * w.cols * 9 // 16 for w in mats)

    def head(self, x: torch.Tensor):
        c = self.cfg
        M = x.shape[0]
        tok, val, key = lm_head_argmax(x, self.lm, softcap=c.softcap, rms_scale=True, eps=c.eps,
                                       row_offset=self.v_rows[0], tokens=self.tokens[:M], values=self.values[:M],
                                       keys=self.keys[:M])
        if self.size > 1:
            key = combine_keys(key, self.group)
        return key, x

    def free(self):
        if getattr(self, "plan", None) is not None:
            self.plan.free()
            self.plan = None
        for L in self.layers:
            for w in L.values():
                w.free()
        self.lm.free()


def norm_weight(seed: int, n: int, device=None) -> torch.Tensor:
    """Seeded synthetic RMSNorm weight: bf16(1 + 0.1 * N(0, 1)), [n]."""
    return (synth_normal(seed, (n,), device=device).float() * 0.1 + 1.0).to(torch.bfloat16)


class DecoderStack:
    """Seeded synthetic weights with the real decoder layer's structure around the quantized linears
    (layer_forward, native_model.cc:899-970, attention left out: q stands in for its output, as in
    SyntheticStack): per layer q|k|v, o, a paired gate|up weight whose phase applies the GeGLU, down,
    the four RMSNorm weights (input, post-attention, pre-feed-forward, post-feed-forward) and the
    layer scalar, then the final norm and the LM head. ``build_plan`` makes the whole step ONE decode
    plan with the norms, residual adds and scalars as phase prologues:

        q|k|v   prologue [post_ffn norm of the previous layer, residual add, its layer scalar]
                then input_layernorm (layer 0: x starts the residual stream)
        o       x = q
        gate|up prologue post_attention_layernorm, residual add, pre_feedforward_layernorm; GeGLU
        down    x = the GeGLU output
        LM head prologue the last layer's post_ffn norm, residual add and scalar, then the final norm

    Tensor parallel like SyntheticStack (q/k/v, gate|up and LM-head rows split, o/down K split with
    the allreduce inside the kernel); the residual stream is kept whole on every rank."""

    def __init__(self, cfg: StackConfig, tp_rank: int = 0, tp_size: int = 1, group=None, max_tokens: int = 8):
        self.cfg, self.rank, self.size, self.group = cfg, tp_rank, tp_size, group
        self.device = torch.device("cuda", torch.cuda.current_device())
        sh = cfg.shapes()
        plan = shard_plan(cfg, tp_rank, tp_size)
        self.q_rows, self.kv_rows, self.i_rows = plan["q_rows"], plan["kv_rows"], plan["i_rows"]
        self.o_cols, self.d_cols, self.v_rows = plan["o_cols"], plan["d_cols"], plan["v_rows"]
        self.nq = self.q_rows[1] - self.q_rows[0]
        self.nkv = self.kv_rows[1] - self.kv_rows[0]
        self.ni = self.i_rows[1] - self.i_rows[0]
        self.max_tokens = max_tokens
        self.layers: List[dict] = []
        i0, i1 = self.i_rows
        for layer in range(cfg.layers):
            mats = {p: synth_matrix(matrix_seed(layer, p), *sh[p]) for p in ("q", "k", "v")}
            qkv = QuantizedWeight.concat([(*mats["q"], self.q_rows), (*mats["k"], self.kv_rows),
                                          (*mats["v"], self.kv_rows)])
            del mats
            o = QuantizedWeight.from_mlx(*synth_matrix(matrix_seed(layer, "o"), *sh["o"]), cols=self.o_cols)
            gate = synth_matrix(matrix_seed(layer, "gate"), *sh["gate"])
            up = synth_matrix(matrix_seed(layer, "up"), *sh["up"])
            gu = QuantizedWeight.geglu_pair(tuple(t[i0:i1] for t in gate), tuple(t[i0:i1] for t in up))
            del gate, up
            down = QuantizedWeight.from_mlx(*synth_matrix(matrix_seed(layer, "down"), *sh["down"]), cols=self.d_cols)
            s = BASE_SEED ^ 0xA000 ^ (layer * 8)
            self.layers.append({"qkv": qkv, "o": o, "gu": gu, "down": down,
                                "in_norm": norm_weight(s, cfg.hidden), "post_attn": norm_weight(s + 1, cfg.hidden),
                                "pre_ffn": norm_weight(s + 2, cfg.hidden), "post_ffn": norm_weight(s + 3, cfg.hidden),
                                "scalar": torch.tensor([1.0 - (layer % 4) / 16], dtype=torch.bfloat16,
                                                       device=self.device)})
        self.lm = QuantizedWeight.from_mlx(*synth_matrix(matrix_seed(0, "lm"), *sh["lm"]), rows=self.v_rows)
        self.final_norm = norm_weight(BASE_SEED ^ 0xAFFF, cfg.hidden)
        dev, M = self.device, max_tokens
        self.tokens = torch.empty(M, dtype=torch.int32, device=dev)
        self.values = torch.empty(M, dtype=torch.float32, device=dev)
        self.keys = torch.empty(M, dtype=torch.int64, device=dev)
        self.plan = None
        torch.cuda.synchronize()

    def build_plan(self, M: int = 1, keep_layers: bool = False) -> DecodePlan:
        """The whole step as one plan of M tokens. ``keep_layers``: every layer writes its own output
        buffers and copies of the residual stream (``self.outs[l]`` with qkv, o, act, h, res_a (the
        stream before q|k|v's input norm), res_b (before gate|up's)), so every phase's input and
        output stay readable after the step; the kernel's work and dataflow are the same."""
        c = self.cfg
        if self.plan is not None:
            self.plan.free()
        if M > self.max_tokens:
            raise ValueError("M above the stack's max_tokens")
        bf = dict(dtype=torch.bfloat16, device=self.device)
        self.h_in = torch.zeros((M, c.hidden), **bf)
        shared = None if keep_layers else {
            "qkv": torch.empty((M, self.nq + 2 * self.nkv), **bf), "o": torch.empty((M, c.hidden), **bf),
            "act": torch.empty((M, self.ni), **bf), "h": torch.empty((M, c.hidden), **bf)}
        self.outs = []
        phases, pro, x = [], [], self.h_in
        ar = PHASE_ALLREDUCE if self.size > 1 else 0
        for i, L in enumerate(self.layers):
            if keep_layers:
                b = {"qkv": torch.empty((M, self.nq + 2 * self.nkv), **bf), "o": torch.empty((M, c.hidden), **bf),
                     "act": torch.empty((M, self.ni), **bf), "h": torch.empty((M, c.hidden), **bf),
                     "res_a": torch.empty((M, c.hidden), **bf), "res_b": torch.empty((M, c.hidden), **bf)}
                self.outs.append(b)
            else:
                b = shared
            if i == 0:
                pro.append({"residual": 1, "norm_weight": L["in_norm"], "residual_out": b.get("res_a"),
                            "eps": c.eps})
            else:
                P = self.layers[i - 1]
                pro.append({"post_norm_weight": P["post_ffn"], "residual": 2, "layer_scalar": P["scalar"],
                            "norm_weight": L["in_norm"], "residual_out": b.get("res_a"), "eps": c.eps})
            phases.append((L["qkv"], x, b["qkv"], 0))
            pro.append(None)
            phases.append((L["o"], b["qkv"][:, : self.nq], b["o"], ar))
            pro.append({"post_norm_weight": L["post_attn"], "residual": 2, "norm_weight": L["pre_ffn"],
                        "residual_out": b.get("res_b"), "eps": c.eps})
            phases.append((L["gu"], b["o"], b["act"], PHASE_GEGLU))
            pro.append(None)
            phases.append((L["down"], b["act"], b["h"], ar))
            x = b["h"]
        P = self.layers[-1]
        self.res_final = torch.empty((M, c.hidden), **bf)
        pro.append({"post_norm_weight": P["post_ffn"], "residual": 2, "layer_scalar": P["scalar"],
                    "norm_weight": self.final_norm, "residual_out": self.res_final, "eps": c.eps})
        phases.append((self.lm, x, None, PHASE_ARGMAX))
        self.plan = DecodePlan(phases, M, rank=self.rank, n_ranks=self.size, group=self.group, prologues=pro)
        self.plan_tokens = M
        return self.plan

    def decode(self, h: torch.Tensor, logits: Optional[torch.Tensor] = None):
        """One step: h [M, hidden] (the plan's M) -> the M greedy keys (LM-head logits into ``logits``,
        bf16 [M, vocab shard], when given)."""
        M = h.shape[0]
        self.h_in[:M].copy_(h)
        self.plan.run(M, softcap=self.cfg.softcap, row_offset=self.v_rows[0], tokens=self.tokens[:M],
                      values=self.values[:M], keys=self.keys[:M], logits=logits)
        return self.keys[:M]

    def local_weight_bytes(self) -> int:
        mats = [w for L in self.layers for k, w in L.items() if k in ("qkv", "o", "gu", "down")] + [self.lm]
        return sum(w.rows * w.cols * 9 // 16 for w in mats)

    def free(self):
        if self.plan is not None:
            self.plan.free()
            self.plan = None
        for L in self.layers:
            for k in ("qkv", "o", "gu", "down"):
                L[k].free()
        self.lm.free()


def decode_keys(keys: torch.Tensor):
    """(token, value) per 64-bit argmax key (inverse of the kernel's key encoding)."""
    k = keys.to(torch.int64).cpu()
    tokens, values = [], []
    for v in k.tolist():
        u = v & (2 ** 64 - 1)
        idx = 0xFFFFFFFF - (u & 0xFFFFFFFF)
        o = u >> 32
        bits = (o & 0x7FFFFFFF) if (o & 0x80000000) else (~o & 0xFFFFFFFF)
        tokens.append(idx)
        values.append(struct.unpack("<f", struct.pack("<I", bits))[0])
    return tokens, values
