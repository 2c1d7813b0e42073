"""GPU, one device: failure detection without a fault. A tensor-parallel decode plan is built as
rank 0 of 2, but its "peer" buffers are local scratch that nothing writes, so the wait for rank 1's
allreduce partial (and for its argmax key) can never be met. Every in-kernel wait is bounded: the
kernel gives up after about two seconds, records a code in the device error word and runs to its
end; the host reads the code, and the context stays usable for the next call."""
import ctypes
import time

import pytest
import torch

from gpu_util import assert_qmm_close, u16

pytestmark = pytest.mark.gpu


def test_tp_plan_wait_runs_out_without_a_peer(cuda, oracle):
    from helios_b200 import _lib
    from helios_b200 import quantized as Q
    assert _lib.device_error() == 0
    w1 = Q.QuantizedWeight.from_mlx(*Q.synth_matrix(11, 4096, 3840))   # every phase fills the grid
    w2 = Q.QuantizedWeight.from_mlx(*Q.synth_matrix(12, 3840, 4096))
    x = Q.synth_normal(13, (1, 3840))
    y1 = torch.empty((1, 4096), dtype=torch.bfloat16, device=cuda)
    y2 = torch.empty((1, 3840), dtype=torch.bfloat16, device=cuda)
    ph = (_lib.G4qDecodePhase * 2)()
    for i, (w, xi, yi, fl) in enumerate(((w1, x, y1, Q.PHASE_ALLREDUCE), (w2, y1, y2, 0))):
        ph[i].weight, ph[i].x, ph[i].ldx = w.handle, xi.data_ptr(), xi.stride(0)
        ph[i].y, ph[i].ldy, ph[i].flags = yi.data_ptr(), yi.stride(0), fl
    plan = ctypes.c_void_p()
    _lib.call("g4q_decode_plan_create_tp", ph, 2, 1, 0, 2, ctypes.byref(plan))
    slots, xkeys = ctypes.c_void_p(), ctypes.c_void_p()
    sb, kb = ctypes.c_uint64(), ctypes.c_uint64()
    _lib.call("g4q_decode_plan_buffers", plan, ctypes.byref(slots), ctypes.byref(sb), ctypes.byref(xkeys),
              ctypes.byref(kb))
    # stand-ins for rank 1's buffers: the plan's sends land here, and nothing ever writes rank 1's
    # partials or key into this rank's buffers
    fake_slots = torch.zeros(sb.value // 8 + 8, dtype=torch.int64, device=cuda)
    fake_keys = torch.zeros(kb.value // 8 + 8, dtype=torch.int64, device=cuda)
    peers = (ctypes.c_void_p * 2)(slots.value, fake_slots.data_ptr())
    keys = (ctypes.c_void_p * 2)(xkeys.value, fake_keys.data_ptr())
    _lib.call("g4q_decode_plan_set_peers", plan, peers, keys)
    torch.cuda.synchronize()
    t0 = time.time()
    _lib.call("g4q_decode_plan_run", plan, 1, 1e-6, 0.0, 0, None, None, None, None, 0,
              ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    elapsed = time.time() - t0
    code = _lib.device_error()           # read and cleared
    _lib.call("g4q_decode_plan_free", plan)
    assert code in (35, 36), f"expected a given-up wait, got device error word {code}"
    assert elapsed < 60
    assert _lib.device_error() == 0
    # the context is still usable: an ordinary matmul right after is correct
    ye, _ = oracle.qmm(u16(x), *oracle.synth_matrix(11, 4096, 3840))
    yf = Q.quantized_matmul(x, w1, out_dtype=torch.float32)
    assert_qmm_close(yf.cpu().numpy(), ye, bf16_out=False)
    assert _lib.device_error() == 0
    w1.free()
    w2.free()
