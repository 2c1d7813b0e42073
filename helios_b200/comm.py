"""Tensor-parallel allreduce over NVLink peer memory (libg4q's g4q_comm_* / g4q_allreduce).

One process per GPU. ``Comm`` creates the rank's exchange buffer, swaps CUDA IPC handles with the
other ranks over a ``torch.distributed`` process group (host-side plumbing only), and then sums
bf16 or fp32 CUDA tensors across the ranks in place: fp32 sums in rank order, the same bits on
every rank. It stands where the Megatron split of the reference's linears needs the sum after
o_proj and down_proj (the reference itself runs one process per model).
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib


class Comm:
    def __init__(self, rank: int, n_ranks: int, max_elems: int, group=None):
        self.rank, self.n_ranks, self.max_elems = rank, n_ranks, max_elems
        self.device = torch.cuda.current_device()
        self._h = ctypes.c_void_p()
        self._opened = []
        _lib.call("g4q_comm_create", rank, n_ranks, max_elems, ctypes.byref(self._h))
        if n_ranks > 1:
            self._connect(group)

    def _connect(self, group):
        buf, nbytes = ctypes.c_void_p(), ctypes.c_uint64()
        _lib.call("g4q_comm_buffer", self._h, ctypes.byref(buf), ctypes.byref(nbytes))
        h = (ctypes.c_uint8 * _lib.IPC_HANDLE_BYTES)()
        _lib.call("g4q_ipc_handle", buf, h)
        handles = [None] * self.n_ranks
        torch.distributed.all_gather_object(handles, bytes(h), group=group)
        peers = (ctypes.c_void_p * self.n_ranks)()
        for r in range(self.n_ranks):
            if r == self.rank:
                peers[r] = buf.value
                continue
            hr = (ctypes.c_uint8 * _lib.IPC_HANDLE_BYTES).from_buffer_copy(handles[r])
            p = ctypes.c_void_p()
            _lib.call("g4q_ipc_open", hr, ctypes.byref(p))
            self._opened.append(p)
            peers[r] = p.value
        _lib.call("g4q_comm_set_peers", self._h, peers)

    def allreduce(self, t: torch.Tensor) -> torch.Tensor:
        """Sum ``t`` (a contiguous bf16 or fp32 CUDA tensor) across the ranks, in place."""
        if t.dtype not in (torch.bfloat16, torch.float32):
            raise ValueError(f"allreduce takes bf16 or fp32 tensors (got {t.dtype})")
        if not t.is_cuda or not t.is_contiguous():
            raise ValueError("allreduce takes a contiguous CUDA tensor")
        dtype = _lib.DTYPE_BF16 if t.dtype == torch.bfloat16 else _lib.DTYPE_F32
        _lib.call("g4q_allreduce", self._h, ctypes.c_void_p(t.data_ptr()), t.numel(), dtype,
                  ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
        return t

    def free(self):
        """Release the communicator; every rank must have finished its calls (e.g. after a barrier)."""
        if self._h:
            torch.cuda.synchronize(self.device)
            for p in self._opened:
                _lib.call("g4q_ipc_close", p)
            self._opened = []
            _lib.call("g4q_comm_free", self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass
