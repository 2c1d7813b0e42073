"""Tensor-parallel host logic on CPU with world_size-2 gloo process groups.

The product's shard plan (row windows for q|k|v, gate|up and the LM head; K windows at group
boundaries for o and down) and its argmax-key combine are exercised with the CPU oracle as the
compute: each rank runs its shards, the fp32 partial sums of o/down are all-reduced, the LM-head
keys are combined with a max, and the result must match the single-process oracle stack. A second
test kills one rank before a collective and checks that the survivor's collective fails within
the process-group timeout instead of hanging (failure detection without any GPU).
"""
import os
import socket
import sys
from datetime import timedelta

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SMALL = dict(layers=2, hidden=256, q_out=256, kv_out=128, inter=512, vocab=2048)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _key(value: np.float32, index: int) -> int:
    """Host restatement of the kernels' argmax key: ordered float bits << 32 | ~index."""
    u = int(np.float32(value).view(np.uint32))
    u = (~u & 0xFFFFFFFF) if (u & 0x80000000) else (u | 0x80000000)
    return (u << 32) | (0xFFFFFFFF - index)


def _tp_worker(rank, world, port, out_q):
    sys.path.insert(0, ROOT)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        from oracle import affine as A
        from helios_b200.stack import StackConfig, combine_keys, shard_plan
        cfg = StackConfig(**SMALL)
        plan = shard_plan(cfg, rank, world)
        sh = A.stack_shapes(cfg.hidden, cfg.q_out, cfg.kv_out, cfg.inter, cfg.vocab)

        def mat(layer, name, rows=None, cols=None):
            w, s, b = A.stack_matrix(layer, name, sh)
            if rows is not None:
                w, s, b = w[rows[0]:rows[1]], s[rows[0]:rows[1]], b[rows[0]:rows[1]]
            if cols is not None:
                w, s, b = w[:, cols[0] // 8:cols[1] // 8], s[:, cols[0] // 64:cols[1] // 64], b[:, cols[0] // 64:cols[1] // 64]
            return [np.ascontiguousarray(a) for a in (w, s, b)]

        def allreduce_f32(y):
            t = torch.from_numpy(y.astype(np.float32))
            dist.all_reduce(t)
            return A.f32_to_bf16(t.numpy())

        h = A.synth_normal_bf16(A.activation_seed(11), cfg.hidden).reshape(1, -1)
        for layer in range(cfg.layers):
            r = np.array([A.rms_scale(h[0], cfg.eps)], dtype=np.float32)
            q = A.qmm(h, *mat(layer, "q", rows=plan["q_rows"]), row_scale=r)[1]
            o = allreduce_f32(A.qmm(q, *mat(layer, "o", cols=plan["o_cols"]))[0])
            r2 = np.array([A.rms_scale(o[0], cfg.eps)], dtype=np.float32)
            up = A.qmm(o, *mat(layer, "up", rows=plan["i_rows"]), row_scale=r2)[1]
            h = allreduce_f32(A.qmm(up, *mat(layer, "down", cols=plan["d_cols"]))[0])
        r3 = np.array([A.rms_scale(h[0], cfg.eps)], dtype=np.float32)
        logits = A.qmm(h, *mat(0, "lm", rows=plan["v_rows"]), row_scale=r3)[1][0]
        t, v = A.softcap_argmax(logits, cfg.softcap)
        key = _key(np.float32(v), plan["v_rows"][0] + t)
        k = combine_keys(torch.tensor([key - (1 << 64) if key >= (1 << 63) else key], dtype=torch.int64))
        kk = int(k.item()) & ((1 << 64) - 1)
        if rank == 0:
            out_q.put((0xFFFFFFFF - (kk & 0xFFFFFFFF), h))
    finally:
        dist.destroy_process_group()


def test_tensor_parallel_decomposition_matches_single_process(oracle):
    ctx = mp.get_context("spawn")
    q = ctx.SimpleQueue()
    port = _free_port()
    mp.start_processes(_tp_worker, args=(2, port, q), nprocs=2, join=True, start_method="spawn")
    token, h = q.get()
    from helios_b200.stack import StackConfig
    cfg = StackConfig(**SMALL)
    ref = oracle.stack_forward(oracle.synth_normal_bf16(oracle.activation_seed(11), cfg.hidden).reshape(1, -1),
                               cfg.layers, oracle.stack_shapes(cfg.hidden, cfg.q_out, cfg.kv_out, cfg.inter, cfg.vocab))
    a, b = oracle.bf16_to_f32(h), oracle.bf16_to_f32(ref["hidden"])
    rms = float(np.sqrt((b.astype(np.float64) ** 2).mean()))
    assert np.abs(a - b).max() <= 2e-2 * rms
    if token != ref["tokens"][0]:
        # a different index is only acceptable on a tie of the softcapped value
        assert abs(oracle.softcap_argmax(ref["logits"][0])[1] - ref["values"][0]) == 0


def test_shard_plan_windows_cover_each_dimension_once():
    sys.path.insert(0, ROOT)
    from helios_b200.stack import StackConfig, shard_plan
    cfg = StackConfig()
    for world in (1, 2, 4, 8):
        plans = [shard_plan(cfg, r, world) for r in range(world)]
        for key, full, align in (("q_rows", cfg.q_out, 16), ("kv_rows", cfg.kv_out, 16), ("i_rows", cfg.inter, 16),
                                 ("v_rows", cfg.vocab, 16), ("o_cols", cfg.q_out, 64), ("d_cols", cfg.inter, 64)):
            spans = [p[key] for p in plans]
            assert spans[0][0] == 0 and spans[-1][1] == full
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            assert all((s1 - s0) % align == 0 for s0, s1 in spans)
    with pytest.raises(ValueError):
        shard_plan(StackConfig(q_out=4096 + 16), 0, 8)


def _dying_worker(rank, world, port, out_q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=5))
    if rank == 1:
        os._exit(0)            # the rank disappears between steps, with no collective in flight
    t = torch.ones(4)
    try:
        dist.all_reduce(t)
        out_q.put("completed")
    except Exception as e:     # gloo reports the lost peer or the timeout
        out_q.put(f"error: {type(e).__name__}")


def test_lost_rank_is_detected_not_hung():
    ctx = mp.get_context("spawn")
    q = ctx.SimpleQueue()
    port = _free_port()
    procs = [ctx.Process(target=_dying_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert not p.is_alive(), "a rank hung instead of failing"
    assert q.get().startswith("error")
