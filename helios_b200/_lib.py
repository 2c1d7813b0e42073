"""ctypes binding of libg4q.so (include/g4q.h).

The product path has no fallback: if the library is missing or cannot load, every call
raises ``G4qUnavailable`` instead of computing anything another way.
"""
from __future__ import annotations

import ctypes
import threading
from pathlib import Path

PKG = Path(__file__).resolve().parent
LIB_PATH = PKG / "libg4q.so"

G4Q_OK = 0
G4Q_ERR_INVALID_ARGUMENT = 1
G4Q_ERR_UNSUPPORTED_CONFIG = 2
G4Q_ERR_MODEL_LOAD = 3
G4Q_ERR_RUNTIME = 4
G4Q_ERR_MEMORY_GUARD = 5
STATUS_NAMES = {
    0: "G4Q_OK",
    1: "G4Q_ERR_INVALID_ARGUMENT",
    2: "G4Q_ERR_UNSUPPORTED_CONFIG",
    3: "G4Q_ERR_MODEL_LOAD",
    4: "G4Q_ERR_RUNTIME",
    5: "G4Q_ERR_MEMORY_GUARD",
}

CHAIN_R1 = 1
CHAIN_R2 = 2
QMM_RMS_SCALE = 0x1
QMM_OUT_F32 = 0x2

# every symbol include/g4q.h declares: name -> (restype, argtypes)
_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_I32 = ctypes.c_int32
_U32 = ctypes.c_uint32
_U64 = ctypes.c_uint64
_F = ctypes.c_float


class G4qVersionInfo(ctypes.Structure):
    _fields_ = [("abi_version", ctypes.c_uint32), ("backend_name", ctypes.c_char_p),
                ("backend_version", ctypes.c_char_p)]


class G4qWeightInfo(ctypes.Structure):
    _fields_ = [("rows", ctypes.c_int64), ("cols", ctypes.c_int64), ("bits", ctypes.c_int32),
                ("group_size", ctypes.c_int32), ("device_bytes", ctypes.c_uint64), ("device", ctypes.c_int32),
                ("fast_path_ok", ctypes.c_int32), ("error_flags", ctypes.c_int32)]


class G4qDecodePhase(ctypes.Structure):
    _fields_ = [("weight", ctypes.c_void_p), ("x", ctypes.c_void_p), ("ldx", ctypes.c_int64), ("y", ctypes.c_void_p),
                ("ldy", ctypes.c_int64), ("flags", ctypes.c_uint32)]


class G4qPhasePrologue(ctypes.Structure):
    _fields_ = [("post_norm_weight", ctypes.c_void_p), ("residual", ctypes.c_int32),
                ("layer_scalar", ctypes.c_void_p), ("norm_weight", ctypes.c_void_p),
                ("residual_out", ctypes.c_void_p), ("ld_residual_out", ctypes.c_int64), ("eps", ctypes.c_float)]


DTYPE_BF16 = 0
DTYPE_F32 = 1
PHASE_ARGMAX = 0x4
PHASE_ALLREDUCE = 0x8
PHASE_GEGLU = 0x10
PATH_GEMV_STREAMK = 1
PATH_GEMV_CLUSTER = 2
PATH_GEMM = 3
PATH_GENERIC = 4
IPC_HANDLE_BYTES = 64

SIGNATURES = {
    "g4q_runtime_version": [ctypes.POINTER(G4qVersionInfo)],
    "g4q_get_last_error": [ctypes.c_char_p, ctypes.c_size_t],
    "g4q_weight_create": [_I64, _I64, _I32, _I32, ctypes.POINTER(_P)],
    "g4q_weight_load": [_P, _I64, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _P],
    "g4q_weight_free": [_P],
    "g4q_weight_info": [_P, ctypes.POINTER(G4qWeightInfo)],
    "g4q_weight_export": [_P, _P, _P, _P, _P],
    "g4q_weight_save": [_P, ctypes.c_char_p],
    "g4q_weight_open": [ctypes.c_char_p, ctypes.POINTER(_P)],
    "g4q_dequantize": [_P, _P, _I64, _P, _I32, _P],
    "g4q_dequantize_mlx": [_P, _P, _P, _I64, _I64, _I32, _I32, _I32, _P, _P],
    "g4q_qmm": [_P, _P, _I64, _I64, _P, _I64, _P],
    "g4q_qmm_ex": [_P, _P, _I64, _I64, _P, _I64, _U32, _F, _P],
    "g4q_qmm_path": [_P, _I64, ctypes.POINTER(_I32), ctypes.POINTER(_I32)],
    "g4q_qmm_norm": [_P, _P, _I64, _I64, _P, _F, _P, _I64, _P, _I64, _P],
    "g4q_qmm_geglu": [_P, _P, _I64, _I64, _P, _U32, _F, _P, _P, _I64, _P],
    "g4q_lm_head_argmax": [_P, _P, _I64, _I64, _F, _U32, _F, _I64, _P, _I64, _P, _P, _P, _P],
    "g4q_lm_head_argmax_noalloc": [_P, _P, _I64, _I64, _P, _I64, _I64, _F, _U32, _F, _I64, _P, _I64, _P, _P, _P, _P],
    "g4q_lora_create": [_I64, _I64, _I32, _F, _P, _P, _I32, ctypes.POINTER(_P)],
    "g4q_lora_apply": [_P, _P, _I64, _I64, _P, _I64, _P],
    "g4q_lora_free": [_P],
    "g4q_geglu": [_P, _I64, _P, _I64, _I64, _I64, _P, _I64, _P],
    "g4q_rms_norm": [_P, _I64, _P, _I64, _I64, _F, _P, _I64, _P],
    "g4q_rms_norm_residual": [_P, _I64, _P, _I64, _I64, _F, _P, _I64, _P, _P, _I64, _P],
    "g4q_device_error": [ctypes.POINTER(_I32), _I32],
    "g4q_decode_plan_create": [ctypes.POINTER(G4qDecodePhase), _I32, _I32, ctypes.POINTER(_P)],
    "g4q_decode_plan_run": [_P, _I64, _F, _F, _I64, _P, _P, _P, _P, _I64, _P],
    "g4q_decode_plan_free": [_P],
    "g4q_decode_plan_trace": [_P, _P, ctypes.POINTER(_I64)],
    "g4q_decode_plan_create_ex": [ctypes.POINTER(G4qDecodePhase), ctypes.POINTER(G4qPhasePrologue), _I32, _I32, _I32,
                                  _I32, ctypes.POINTER(_P)],
    "g4q_decode_plan_create_tp": [ctypes.POINTER(G4qDecodePhase), _I32, _I32, _I32, _I32, ctypes.POINTER(_P)],
    "g4q_decode_plan_buffers": [_P, ctypes.POINTER(_P), ctypes.POINTER(ctypes.c_uint64), ctypes.POINTER(_P),
                                ctypes.POINTER(ctypes.c_uint64)],
    "g4q_decode_plan_set_peers": [_P, ctypes.POINTER(_P), ctypes.POINTER(_P)],
    "g4q_ipc_handle": [_P, ctypes.POINTER(ctypes.c_uint8)],
    "g4q_ipc_open": [ctypes.POINTER(ctypes.c_uint8), ctypes.POINTER(_P)],
    "g4q_ipc_close": [_P],
    "g4q_comm_create": [_I32, _I32, _I64, ctypes.POINTER(_P)],
    "g4q_comm_buffer": [_P, ctypes.POINTER(_P), ctypes.POINTER(ctypes.c_uint64)],
    "g4q_comm_set_peers": [_P, ctypes.POINTER(_P)],
    "g4q_allreduce": [_P, _P, _I64, _I32, _P],
    "g4q_comm_free": [_P],
    "g4q_synth_matrix": [_U64, _I64, _I64, _I32, _I32, _P, _P, _P, _P],
    "g4q_synth_normal_bf16": [_U64, _I64, _P, _P],
}


class G4qError(RuntimeError):
    """A libg4q call returned a non-OK status; ``status`` and ``message`` carry it."""

    def __init__(self, status: int, message: str, fn: str = ""):
        self.status = status
        self.message = message
        super().__init__(f"{fn or 'g4q'} failed with {STATUS_NAMES.get(status, status)}: {message}")


class G4qInvalidArgument(G4qError, ValueError):
    pass


class G4qUnavailable(RuntimeError):
    """libg4q.so is not built or cannot be loaded; there is no fallback."""


_lib = None
_lock = threading.Lock()


def load(path: Path | None = None):
    global _lib
    with _lock:
        if _lib is None:
            p = Path(path) if path else LIB_PATH
            if not p.exists():
                raise G4qUnavailable(
                    f"{p} is missing: build it with `python -m helios_b200.build` (nvcc, sm_100a)")
            try:
                L = ctypes.CDLL(str(p))
            except OSError as e:
                raise G4qUnavailable(f"cannot load {p}: {e}") from e
            for name, argtypes in SIGNATURES.items():
                fn = getattr(L, name)
                fn.restype = ctypes.c_int
                fn.argtypes = argtypes
            _lib = L
    return _lib


def last_error() -> str:
    buf = ctypes.create_string_buffer(512)
    load().g4q_get_last_error(buf, 512)
    return buf.value.decode(errors="replace")


def call(name: str, *args) -> None:
    """Call a g4q entry point and raise G4qError on a non-OK status."""
    status = getattr(load(), name)(*args)
    if status != G4Q_OK:
        msg = last_error()
        cls = G4qInvalidArgument if status == G4Q_ERR_INVALID_ARGUMENT else G4qError
        raise cls(status, msg, name)


def device_error(reset: bool = True) -> int:
    """Nonzero when a bounded in-kernel wait gave up since the last reset (results invalid)."""
    code = ctypes.c_int32(0)
    call("g4q_device_error", ctypes.byref(code), 1 if reset else 0)
    return code.value


def version() -> dict:
    info = G4qVersionInfo()
    call("g4q_runtime_version", ctypes.byref(info))
    return {"abi_version": info.abi_version, "backend_name": info.backend_name.decode(),
            "backend_version": info.backend_version.decode()}
