"""Host-side mirror of the MLX affine-quantization operators that Helios's native graph calls.

The reference graph (native/gemma4_mlx/src/native_model.cc) uses exactly these MLX ops on
its weights:

* ``quantized_linear`` (:349-362): ``mlx::core::quantized_matmul(x, W, scales, biases,
  transpose=true, group_size, bits, "affine")`` then a bf16 cast;
* ``quantized_embedding`` (:364-376): ``take`` rows, then ``mlx::core::dequantize``;
* ``target_logits_for_hidden`` (:1782-1795): the tied LM head, bf16 ``tanh(l/30)*30`` softcap,
  followed by ``argmax`` (:3825).

``quantized_matmul`` / ``dequantize`` below keep MLX's names, argument meaning and shape rules
(``w`` is uint32 ``[N, K*bits/32]``, scales/biases ``[N, K/group_size]``, ``transpose=True``
computes ``x @ dequantize(w).T``) and raise ``ValueError`` on bad arguments as MLX does. All
compute runs in libg4q.so (sm_100a kernels) on the current CUDA stream; tensors are torch
CUDA tensors. There is no CPU path.
"""
from __future__ import annotations

import ctypes
from typing import Optional, Tuple

import torch

from . import _lib
from ._lib import (CHAIN_R1, CHAIN_R2, PHASE_ALLREDUCE, PHASE_ARGMAX, PHASE_GEGLU, QMM_OUT_F32, QMM_RMS_SCALE,
                   G4qError, G4qInvalidArgument)

__all__ = [
    "QuantizedWeight", "quantized_matmul", "quantized_linear", "norm_quantized_matmul", "quantized_matmul_geglu",
    "LoraAdapter", "geglu", "rms_norm", "rms_norm_residual", "dequantize", "lm_head_argmax", "DecodePlan",
    "synth_matrix", "synth_normal", "CHAIN_R1", "CHAIN_R2", "QMM_RMS_SCALE", "QMM_OUT_F32", "PHASE_ARGMAX",
    "PHASE_ALLREDUCE", "PHASE_GEGLU", "G4qError", "G4qInvalidArgument",
]


def _stream() -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _ptr(t: Optional[torch.Tensor]) -> Optional[ctypes.c_void_p]:
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _as_bits16(t: torch.Tensor, name: str) -> torch.Tensor:
    if t.dtype in (torch.bfloat16, torch.int16, torch.uint16):
        return t
    raise ValueError(f"{name} must be bfloat16 (got {t.dtype})")


def _check_format(group_size: int, bits: int, mode: str) -> None:
    if mode != "affine":
        raise ValueError(f"[quantize] only mode='affine' is supported (got {mode!r})")
    if bits not in (4, 8):
        raise ValueError(f"[quantize] bits must be 4 or 8 (got {bits})")
    if group_size not in (32, 64, 128):
        raise ValueError(f"[quantize] group_size must be 32, 64 or 128 (got {group_size})")


class QuantizedWeight:
    """An affine-quantized matrix resident on one GPU.

    4-bit group-64 matrices (every projection of the default manifest) are repacked into libg4q's
    kernel layout and run on the tensor-core / persistent kernels; the 8-bit group-64 per-module
    override a manifest may name (model_manifest.cc:146-152), and groups 32 / 128, stay in MLX's
    layout and run on the generic kernels (quantized matmul and dequantize only: the fused LM
    head and the decode plan reject them). Build it from MLX-layout tensors (host or device) with :meth:`from_mlx`, optionally
    taking a row window (tensor-parallel column split) and/or a group-aligned column window (row
    split), or concatenating several matrices that share an input with :meth:`concat`.
    """

    def __init__(self, rows: int, cols: int, bits: int = 4, group_size: int = 64):
        self._h = ctypes.c_void_p()
        _lib.call("g4q_weight_create", rows, cols, bits, group_size, ctypes.byref(self._h))
        self.rows, self.cols, self.bits, self.group_size = rows, cols, bits, group_size
        self.device = torch.cuda.current_device()

    @property
    def handle(self) -> ctypes.c_void_p:
        if not self._h:
            raise ValueError("QuantizedWeight has been freed")
        return self._h

    @property
    def shape(self) -> Tuple[int, int]:
        return (self.rows, self.cols)

    def load(self, w: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor, *, dst_row: int = 0,
             src_row: int = 0, src_col: int = 0, n_rows: Optional[int] = None) -> "QuantizedWeight":
        if w.dtype not in (torch.uint32, torch.int32):
            raise ValueError(f"w must be uint32 packed words (got {w.dtype})")
        _as_bits16(scales, "scales")
        _as_bits16(biases, "biases")
        if w.dim() != 2 or scales.dim() != 2 or biases.dim() != 2:
            raise ValueError("w, scales and biases must be 2-D")
        src_rows, src_cols = w.shape[0], w.shape[1] * 32 // self.bits
        if scales.shape != (src_rows, src_cols // self.group_size) or biases.shape != scales.shape:
            raise ValueError(f"scales/biases must be [{src_rows}, {src_cols // self.group_size}] "
                             f"(got {tuple(scales.shape)}, {tuple(biases.shape)})")
        w, scales, biases = w.contiguous(), scales.contiguous(), biases.contiguous()
        n = self.rows - dst_row if n_rows is None else n_rows
        _lib.call("g4q_weight_load", self.handle, dst_row, _ptr(w), _ptr(scales), _ptr(biases), src_rows,
                  src_cols, src_row, src_col, n, _stream())
        return self

    @classmethod
    def from_mlx(cls, w: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor, *, group_size: int = 64,
                 bits: int = 4, rows: Optional[Tuple[int, int]] = None,
                 cols: Optional[Tuple[int, int]] = None) -> "QuantizedWeight":
        """Upload an MLX-layout matrix; ``rows=(start, stop)`` / ``cols=(start, stop)`` take a window."""
        src_rows, src_cols = w.shape[0], w.shape[1] * 32 // bits
        r0, r1 = rows if rows is not None else (0, src_rows)
        c0, c1 = cols if cols is not None else (0, src_cols)
        q = cls(r1 - r0, c1 - c0, bits, group_size)
        return q.load(w, scales, biases, src_row=r0, src_col=c0)

    @classmethod
    def concat(cls, parts, *, group_size: int = 64, bits: int = 4) -> "QuantizedWeight":
        """Stack several (w, scales, biases[, (row0, row1)]) MLX-layout matrices along N."""
        spans, cols = [], None
        for p in parts:
            w = p[0]
            r0, r1 = p[3] if len(p) > 3 and p[3] is not None else (0, w.shape[0])
            c = w.shape[1] * 32 // bits
            if cols is not None and c != cols:
                raise ValueError("concatenated matrices must share K")
            cols = c
            spans.append((p, r0, r1))
        q = cls(sum(r1 - r0 for _, r0, r1 in spans), cols, bits, group_size)
        dst = 0
        for p, r0, r1 in spans:
            q.load(p[0], p[1], p[2], dst_row=dst, src_row=r0, n_rows=r1 - r0)
            dst += r1 - r0
        return q

    @classmethod
    def geglu_pair(cls, gate, up) -> "QuantizedWeight":
        """A paired gate|up weight for :func:`quantized_matmul_geglu`: gate and up are MLX-layout
        (w, scales, biases) triples of the same [I, K] shape (I % 32 == 0); the upload interleaves
        them in 32-row slices, so each 64-row quad holds 32 gate rows and the same 32 up rows."""
        parts = []
        for a, b in zip(gate, up):
            if a.shape != b.shape or a.shape[0] % 32 != 0:
                raise ValueError("gate and up must have the same shape with rows a multiple of 32")
            n = a.shape[0]
            parts.append(torch.stack([a.reshape(n // 32, 32, -1), b.reshape(n // 32, 32, -1)], dim=1)
                         .reshape(2 * n, -1))
        return cls.from_mlx(*parts)

    def save(self, path) -> None:
        """Write the repacked buffers to a versioned cache file (g4q_weight_save)."""
        _lib.call("g4q_weight_save", self.handle, str(path).encode())

    @classmethod
    def open(cls, path) -> "QuantizedWeight":
        """A handle on the current GPU from a cache file written by :meth:`save`, without a repack."""
        q = cls.__new__(cls)
        q._h = ctypes.c_void_p()
        _lib.call("g4q_weight_open", str(path).encode(), ctypes.byref(q._h))
        info = _lib.G4qWeightInfo()
        _lib.call("g4q_weight_info", q._h, ctypes.byref(info))
        q.rows, q.cols, q.bits, q.group_size = info.rows, info.cols, info.bits, info.group_size
        q.device = torch.cuda.current_device()
        return q

    def info(self) -> dict:
        info = _lib.G4qWeightInfo()
        _lib.call("g4q_weight_info", self.handle, ctypes.byref(info))
        return {f: getattr(info, f) for f, _ in info._fields_}

    def qmm_path(self, M: int) -> Tuple[int, int]:
        """(kernel, splits) that quantized_matmul takes at M rows (``_lib.PATH_*``; splits is the
        GEMM's k-block split count, 0 for the other kernels). Launches nothing."""
        kernel, splits = ctypes.c_int32(0), ctypes.c_int32(0)
        _lib.call("g4q_qmm_path", self.handle, M, ctypes.byref(kernel), ctypes.byref(splits))
        return kernel.value, splits.value

    def export(self) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
        """Inverse repack: MLX-layout (w uint32, scales bf16, biases bf16) on this GPU."""
        dev = torch.device("cuda", self.device)
        w = torch.empty((self.rows, self.cols * self.bits // 32), dtype=torch.uint32, device=dev)
        s = torch.empty((self.rows, self.cols // self.group_size), dtype=torch.bfloat16, device=dev)
        b = torch.empty_like(s)
        _lib.call("g4q_weight_export", self.handle, _ptr(w), _ptr(s), _ptr(b), _stream())
        return w, s, b

    def free(self) -> None:
        if self._h:
            _lib.call("g4q_weight_free", self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


def _rows2d(x: torch.Tensor, K: int, name: str = "x") -> torch.Tensor:
    if x.dtype != torch.bfloat16:
        raise ValueError(f"{name} must be bfloat16 (got {x.dtype})")
    if not x.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor")
    if x.shape[-1] != K:
        raise ValueError(f"[quantized_matmul] last dimension of {name} ({x.shape[-1]}) must equal K = {K}")
    x2 = x.reshape(-1, K)
    if x2.stride(1) != 1 or x2.stride(0) % 8 != 0 or x2.data_ptr() % 16 != 0:
        x2 = x2.contiguous()
    return x2


def quantized_matmul(x: torch.Tensor, w, scales: Optional[torch.Tensor] = None,
                     biases: Optional[torch.Tensor] = None, transpose: bool = True, group_size: int = 64,
                     bits: int = 4, mode: str = "affine", *, rms_scale: bool = False, eps: float = 1e-6,
                     out_dtype: torch.dtype = torch.bfloat16, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``x @ dequantize(w).T`` with fp32 accumulation and bf16 (or fp32) output.

    ``w`` is a :class:`QuantizedWeight` (scales/biases None) or MLX-layout tensors (uploaded per
    call; use a QuantizedWeight for repeated calls). ``rms_scale`` folds the input RMSNorm
    ``1/sqrt(mean(x^2)+eps)`` into the output.
    """
    _check_format(group_size, bits, mode)
    if not transpose:
        raise ValueError("[quantized_matmul] only transpose=True (x @ W.T) is on the Helios path")
    if isinstance(w, QuantizedWeight):
        if scales is not None or biases is not None:
            raise ValueError("scales/biases are part of a QuantizedWeight")
        qw = w
    else:
        if scales is None or biases is None:
            raise ValueError("[quantized_matmul] affine mode needs scales and biases")
        qw = QuantizedWeight.from_mlx(w, scales, biases, group_size=group_size, bits=bits)
    if (qw.group_size, qw.bits) != (group_size, bits):
        raise ValueError("group_size/bits do not match the uploaded weight")
    x2 = _rows2d(x, qw.cols)
    M = x2.shape[0]
    if out_dtype not in (torch.bfloat16, torch.float32):
        raise ValueError("out_dtype must be bfloat16 or float32")
    shape = tuple(x.shape[:-1]) + (qw.rows,)
    y = torch.empty(shape, dtype=out_dtype, device=x.device) if out is None else out
    if y.dtype != out_dtype or y.shape[-1] != qw.rows:
        raise ValueError("out has the wrong dtype or shape")
    y2 = y.view(-1, qw.rows) if y.is_contiguous() else None
    if y2 is None:
        raise ValueError("out must be contiguous")
    flags = (QMM_RMS_SCALE if rms_scale else 0) | (QMM_OUT_F32 if out_dtype == torch.float32 else 0)
    _lib.call("g4q_qmm_ex", qw.handle, _ptr(x2), M, x2.stride(0), _ptr(y2), y2.stride(0), flags, eps, _stream())
    return y


class LoraAdapter:
    """One LoRA adapter module on one GPU (NativeLoraAdapter::Impl::Module, native_model.cc:66-73).

    ``lora_a`` is ``[rank, in_features]`` and ``lora_b`` ``[out_features, rank]`` as the adapter's
    safetensors store them (``*.lora_A.weight`` / ``*.lora_B.weight``), any float dtype, host or
    device; they are converted to fp32 as at native_model.cc:3419-3420 and the scale is
    ``alpha / rank`` (:3378). Validation as in NativeLoraAdapter::load (:3332-3339, :3399-3411):
    rank > 0, alpha finite and positive, shapes consistent. ``max_tokens`` sizes the low-rank
    scratch; longer inputs are processed in chunks of it.
    """

    def __init__(self, lora_a: torch.Tensor, lora_b: torch.Tensor, alpha: float, *, max_tokens: int = 2048):
        if lora_a.dim() != 2 or lora_b.dim() != 2:
            raise ValueError("LoRA tensors must be rank-2")
        rank, cols = lora_a.shape
        rows = lora_b.shape[0]
        if lora_b.shape[1] != rank:
            raise ValueError(f"LoRA shape mismatch: A=[{rank},{cols}] B=[{rows},{lora_b.shape[1]}]")
        a = lora_a.detach().to(torch.float32).contiguous()
        b = lora_b.detach().to(torch.float32).contiguous()
        self._h = ctypes.c_void_p()
        _lib.call("g4q_lora_create", rows, cols, rank, float(alpha), _ptr(a), _ptr(b), max_tokens,
                  ctypes.byref(self._h))
        self.rows, self.cols, self.rank, self.alpha = rows, cols, rank, float(alpha)
        self.device = torch.cuda.current_device()

    @property
    def handle(self) -> ctypes.c_void_p:
        if not self._h:
            raise ValueError("LoraAdapter has been freed")
        return self._h

    def apply(self, x: torch.Tensor, y: torch.Tensor) -> torch.Tensor:
        """In place: ``y = bf16(y + bf16((f32(x) @ A.T @ B.T) * bf16(alpha/rank)))`` (native_model.cc:316-328)."""
        x2 = _rows2d(x, self.cols)
        if y.dtype != torch.bfloat16 or not y.is_contiguous() or y.shape[-1] != self.rows:
            raise ValueError("y must be a contiguous bfloat16 tensor with last dimension = out_features")
        y2 = y.view(-1, self.rows)
        if y2.shape[0] != x2.shape[0]:
            raise ValueError("x and y must have the same number of rows")
        _lib.call("g4q_lora_apply", self.handle, _ptr(x2), x2.shape[0], x2.stride(0), _ptr(y2), y2.stride(0),
                  _stream())
        return y

    def free(self) -> None:
        if self._h:
            _lib.call("g4q_lora_free", self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


def quantized_linear(x: torch.Tensor, w: QuantizedWeight, lora: Optional[LoraAdapter] = None) -> torch.Tensor:
    """quantized_linear (native_model.cc:349-362): the affine quantized matmul, bf16 output, then the
    adapter's delta when one is active for this module (add_lora_delta_if_active, :316-328)."""
    y = quantized_matmul(x, w, group_size=w.group_size, bits=w.bits)
    if lora is not None:
        if (lora.rows, lora.cols) != (w.rows, w.cols):
            raise ValueError("the LoRA module's shape does not match the weight")
        lora.apply(x, y)
    return y


def _bf16_rows(t: torch.Tensor, name: str) -> torch.Tensor:
    if t.dtype != torch.bfloat16 or not t.is_cuda:
        raise ValueError(f"{name} must be a bfloat16 CUDA tensor")
    t2 = t.reshape(-1, t.shape[-1])
    if t2.stride(1) != 1 or t2.stride(0) % 8 != 0 or t2.data_ptr() % 16 != 0:
        t2 = t2.contiguous()
    return t2


def geglu(gate: torch.Tensor, up: torch.Tensor, *, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """geglu (native_model.cc:378-386): bf16 ``0.5*g*(1 + tanh(sqrt(2/pi)*(g + 0.044715*g^3))) * up``
    with the reference's nine bf16 roundings, in one kernel. ``gate`` and ``up`` may be the two
    halves of one gate|up matmul output (``y[..., :I]``, ``y[..., I:]``)."""
    if gate.shape != up.shape:
        raise ValueError("gate and up must have the same shape")
    I = gate.shape[-1]
    if I % 8 != 0:
        raise ValueError("the last dimension must be a multiple of 8")
    g2, u2 = _bf16_rows(gate, "gate"), _bf16_rows(up, "up")
    res = torch.empty(gate.shape, dtype=torch.bfloat16, device=gate.device) if out is None else out
    o2 = _bf16_rows(res, "out")
    if o2.data_ptr() != res.data_ptr() or o2.shape != g2.shape:
        raise ValueError("out must be a contiguous tensor shaped like gate")
    _lib.call("g4q_geglu", _ptr(g2), g2.stride(0), _ptr(u2), u2.stride(0), g2.shape[0], I, _ptr(o2), o2.stride(0),
              _stream())
    return res


def rms_norm(x: torch.Tensor, weight: Optional[torch.Tensor] = None, eps: float = 1e-6, *,
             out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``model_dtype(mlx::core::fast::rms_norm(x, weight, eps))`` over the last dimension
    (native_model.cc:910-913 and the other norms of a layer): bf16(weight * bf16(x / rms(x)))."""
    K = x.shape[-1]
    if K % 8 != 0:
        raise ValueError("the last dimension must be a multiple of 8")
    x2 = _bf16_rows(x, "x")
    w = None
    if weight is not None:
        if weight.shape != (K,):
            raise ValueError(f"weight must have shape ({K},)")
        w = _bf16_rows(weight.view(1, K), "weight")
    res = torch.empty(x.shape, dtype=torch.bfloat16, device=x.device) if out is None else out
    o2 = _bf16_rows(res, "out")
    if o2.data_ptr() != res.data_ptr() or o2.shape != x2.shape:
        raise ValueError("out must be a contiguous tensor shaped like x")
    _lib.call("g4q_rms_norm", _ptr(x2), x2.stride(0), _ptr(w), x2.shape[0], K, float(eps), _ptr(o2), o2.stride(0),
              _stream())
    return res


def rms_norm_residual(x: torch.Tensor, weight: Optional[torch.Tensor], residual: torch.Tensor,
                      layer_scalar: Optional[torch.Tensor] = None, eps: float = 1e-6, *,
                      out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """The tail of a layer's sub-block (native_model.cc:954-968 / :920-926) in one kernel:
    ``bf16(bf16(residual + rms_norm(x, weight, eps)) * layer_scalar)`` (no scalar when None)."""
    K = x.shape[-1]
    if K % 8 != 0:
        raise ValueError("the last dimension must be a multiple of 8")
    if residual.shape != x.shape:
        raise ValueError("residual must be shaped like x")
    x2, r2 = _bf16_rows(x, "x"), _bf16_rows(residual, "residual")
    w = None
    if weight is not None:
        if weight.shape != (K,):
            raise ValueError(f"weight must have shape ({K},)")
        w = _bf16_rows(weight.view(1, K), "weight")
    sc = None
    if layer_scalar is not None:
        if layer_scalar.numel() != 1 or layer_scalar.dtype != torch.bfloat16 or not layer_scalar.is_cuda:
            raise ValueError("layer_scalar must be one bf16 value on the GPU")
        sc = layer_scalar.reshape(1)
    res = torch.empty(x.shape, dtype=torch.bfloat16, device=x.device) if out is None else out
    o2 = _bf16_rows(res, "out")
    if o2.data_ptr() != res.data_ptr() or o2.shape != x2.shape:
        raise ValueError("out must be a contiguous tensor shaped like x")
    _lib.call("g4q_rms_norm_residual", _ptr(x2), x2.stride(0), _ptr(w), x2.shape[0], K, float(eps), _ptr(r2),
              r2.stride(0), _ptr(sc), _ptr(o2), o2.stride(0), _stream())
    return res


def norm_quantized_matmul(x: torch.Tensor, norm_weight: torch.Tensor, w: QuantizedWeight, *, eps: float = 1e-6,
                          xn: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``quantized_matmul(rms_norm(x, norm_weight, eps), w)`` -- the norm -> linear pair of
    layer_forward (native_model.cc:910-913, 929-932). At M <= 8 the norm is fused into the decode
    GEMV's staging of x (one launch); ``xn``, if given, also receives the normalized rows. Larger M
    needs ``xn`` (bf16, shaped like x): the normalized rows are written there, then multiplied."""
    x2 = _rows2d(x, w.cols)
    M = x2.shape[0]
    if norm_weight.shape != (w.cols,) or norm_weight.dtype != torch.bfloat16:
        raise ValueError(f"norm_weight must be bf16 of shape ({w.cols},)")
    nw = norm_weight.contiguous()
    xn2 = None
    if xn is not None:
        if xn.dtype != torch.bfloat16 or not xn.is_contiguous() or xn.numel() != M * w.cols:
            raise ValueError("xn must be a contiguous bf16 tensor shaped like x")
        xn2 = xn.view(M, w.cols)
    shape = tuple(x.shape[:-1]) + (w.rows,)
    y = torch.empty(shape, dtype=torch.bfloat16, device=x.device) if out is None else out
    if y.dtype != torch.bfloat16 or not y.is_contiguous() or y.shape[-1] != w.rows:
        raise ValueError("out must be a contiguous bf16 tensor with last dimension = rows")
    y2 = y.view(-1, w.rows)
    _lib.call("g4q_qmm_norm", w.handle, _ptr(x2), M, x2.stride(0), _ptr(nw), float(eps), _ptr(xn2),
              0 if xn2 is None else xn2.stride(0), _ptr(y2), y2.stride(0), _stream())
    return y


def quantized_matmul_geglu(x: torch.Tensor, w: QuantizedWeight, *, norm_weight: Optional[torch.Tensor] = None,
                           rms_scale: bool = False, eps: float = 1e-6, y: Optional[torch.Tensor] = None,
                           out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``geglu(x @ gate.T, x @ up.T)`` for a paired gate|up weight (:meth:`QuantizedWeight.geglu_pair`):
    the gate/up projections and the GeGLU of layer_forward (native_model.cc:934-945). At M <= 8 the
    GeGLU runs in the decode GEMV's epilogue; larger M needs ``y`` (bf16 [..., rows]) for the paired
    matmul output. ``norm_weight`` (M <= 8 only) first applies the pre-feed-forward RMSNorm
    (:929-932) in the same launch. Returns bf16 [..., rows / 2]."""
    nw = None
    if norm_weight is not None:
        if norm_weight.shape != (w.cols,) or norm_weight.dtype != torch.bfloat16:
            raise ValueError(f"norm_weight must be bf16 of shape ({w.cols},)")
        nw = norm_weight.contiguous()
    x2 = _rows2d(x, w.cols)
    M = x2.shape[0]
    I = w.rows // 2
    shape = tuple(x.shape[:-1]) + (I,)
    act = torch.empty(shape, dtype=torch.bfloat16, device=x.device) if out is None else out
    if act.dtype != torch.bfloat16 or not act.is_contiguous() or act.shape[-1] != I:
        raise ValueError("out must be a contiguous bf16 tensor with last dimension rows / 2")
    if y is not None and (y.dtype != torch.bfloat16 or not y.is_contiguous() or y.numel() != M * w.rows):
        raise ValueError("y must be a contiguous bf16 tensor of M x rows elements")
    _lib.call("g4q_qmm_geglu", w.handle, _ptr(x2), M, x2.stride(0), _ptr(nw), QMM_RMS_SCALE if rms_scale else 0,
              eps, _ptr(y), _ptr(act), I, _stream())
    return act


def dequantize(w, scales: Optional[torch.Tensor] = None, biases: Optional[torch.Tensor] = None,
               group_size: int = 64, bits: int = 4, mode: str = "affine", *, rows: Optional[torch.Tensor] = None,
               chain: int = CHAIN_R2) -> torch.Tensor:
    """bf16 ``scale * q + bias`` of every element (or of the rows ``rows``, an int32 index tensor).

    ``w`` is a :class:`QuantizedWeight` or MLX-layout device tensors (any of bits 4/8, group
    32/64/128). Bit-exact with rounding chain ``chain`` (R2 default: bf16(bf16(s*q) + b)).
    """
    _check_format(group_size, bits, mode)
    if chain not in (CHAIN_R1, CHAIN_R2):
        raise ValueError("chain must be CHAIN_R1 or CHAIN_R2")
    if isinstance(w, QuantizedWeight):
        dev = torch.device("cuda", w.device)
        if rows is None:
            out = torch.empty((w.rows, w.cols), dtype=torch.bfloat16, device=dev)
            _lib.call("g4q_dequantize", w.handle, None, 0, _ptr(out), chain, _stream())
        else:
            ids = rows.to(device=dev, dtype=torch.int32).contiguous().view(-1)
            out = torch.empty(tuple(rows.shape) + (w.cols,), dtype=torch.bfloat16, device=dev)
            _lib.call("g4q_dequantize", w.handle, _ptr(ids), ids.numel(), _ptr(out), chain, _stream())
        return out
    if scales is None or biases is None:
        raise ValueError("[dequantize] affine mode needs scales and biases")
    if not w.is_cuda:
        raise ValueError("w must be a CUDA tensor")
    N, K = w.shape[0], w.shape[1] * 32 // bits
    if rows is not None:
        ids = rows.to(device=w.device, dtype=torch.long).view(-1)
        w, scales, biases = w[ids], scales[ids], biases[ids]
        N = ids.numel()
    w, scales, biases = w.contiguous(), scales.contiguous(), biases.contiguous()
    if scales.shape != (N, K // group_size) or biases.shape != scales.shape:
        raise ValueError("scales/biases must be [N, K/group_size]")
    out = torch.empty((N, K), dtype=torch.bfloat16, device=w.device)
    _lib.call("g4q_dequantize_mlx", _ptr(w), _ptr(scales), _ptr(biases), N, K, bits, group_size, chain, _ptr(out),
              _stream())
    return out if rows is None else out.view(tuple(rows.shape) + (K,))


def lm_head_argmax(x: torch.Tensor, w: QuantizedWeight, *, softcap: float = 30.0, rms_scale: bool = False,
                   eps: float = 1e-6, row_offset: int = 0, logits: Optional[torch.Tensor] = None,
                   tokens: Optional[torch.Tensor] = None, values: Optional[torch.Tensor] = None,
                   keys: Optional[torch.Tensor] = None):
    """Tied LM head + bf16 softcap + greedy argmax (first index wins ties), one pass over W.

    Returns (tokens int32 [M], values float32 [M], keys int64 [M]); ``logits`` (bf16 [M, N]),
    if given, receives the pre-softcap logits.
    """
    x2 = _rows2d(x, w.cols)
    M = x2.shape[0]
    dev = x.device
    tokens = torch.empty(M, dtype=torch.int32, device=dev) if tokens is None else tokens
    values = torch.empty(M, dtype=torch.float32, device=dev) if values is None else values
    keys = torch.empty(M, dtype=torch.int64, device=dev) if keys is None else keys
    ld = 0
    if logits is not None:
        if logits.dtype != torch.bfloat16 or logits.shape[-1] != w.rows or not logits.is_contiguous():
            raise ValueError("logits must be contiguous bf16 [M, rows]")
        ld = w.rows
    _lib.call("g4q_lm_head_argmax", w.handle, _ptr(x2), M, x2.stride(0), softcap,
              QMM_RMS_SCALE if rms_scale else 0, eps, row_offset, _ptr(logits), ld, _ptr(tokens), _ptr(values),
              _ptr(keys), _stream())
    return tokens, values, keys


class DecodePlan:
    """All quantized matmuls of one decode step as ONE persistent kernel launch (g4q_decode_plan_*).

    ``phases`` is a list of ``(weight, x, y, flags)``: ``x`` a bf16 CUDA tensor view [M, K] (row stride a
    multiple of 8), ``y`` a bf16/fp32 CUDA tensor view [M, N] or None for the final argmax phase;
    ``flags`` from QMM_RMS_SCALE / QMM_OUT_F32 / PHASE_ARGMAX / PHASE_ALLREDUCE / PHASE_GEGLU (a
    paired gate|up weight whose y is the [M, rows / 2] GeGLU). Phase i may read phase i-1's output.
    ``max_tokens``: the tokens of every step, 1, 2, 4 or 8. Tensor addresses are baked into the plan:
    keep the tensors alive and reuse them.

    Tensor parallel: pass ``rank``/``n_ranks`` and the process ``group``; every rank builds the plan of
    its own shards (collectively), the plans exchange their slot buffers by CUDA IPC over the group,
    and ALLREDUCE phases then sum their partials across ranks inside the kernel.
    """

    def __init__(self, phases, max_tokens: int = 1, *, rank: int = 0, n_ranks: int = 1, group=None, prologues=None):
        """``prologues``: None, or one dict (or None) per phase with the keys of G4qPhasePrologue:
        ``post_norm_weight``, ``residual`` (0/1/2), ``layer_scalar``, ``norm_weight`` (bf16 CUDA tensors or
        None), ``residual_out`` (bf16 [M, ld] or None), ``eps``."""
        self._keep = []
        self._opened = []
        arr = (_lib.G4qDecodePhase * len(phases))()
        pro = None
        if prologues is not None:
            if len(prologues) != len(phases):
                raise ValueError("one prologue entry (or None) per phase")
            pro = (_lib.G4qPhasePrologue * len(phases))()
            for i, d in enumerate(prologues):
                d = d or {}
                pro[i].post_norm_weight = _ptr(d.get("post_norm_weight"))
                pro[i].residual = int(d.get("residual", 0))
                pro[i].layer_scalar = _ptr(d.get("layer_scalar"))
                pro[i].norm_weight = _ptr(d.get("norm_weight"))
                ro = d.get("residual_out")
                pro[i].residual_out = _ptr(ro)
                pro[i].ld_residual_out = 0 if ro is None else ro.stride(0)
                pro[i].eps = float(d.get("eps", 1e-6))
                self._keep += [d.get(k) for k in ("post_norm_weight", "layer_scalar", "norm_weight", "residual_out")]
        for i, (w, x, y, flags) in enumerate(phases):
            if x.dtype != torch.bfloat16 or x.stride(-1) != 1:
                raise ValueError(f"phase {i}: x must be a bf16 view with unit column stride")
            arr[i].weight = w.handle
            arr[i].x = x.data_ptr()
            arr[i].ldx = x.stride(0)
            arr[i].y = None if y is None else y.data_ptr()
            arr[i].ldy = 0 if y is None else y.stride(0)
            arr[i].flags = flags
            self._keep += [w, x, y]
        self._h = ctypes.c_void_p()
        if pro is not None:
            _lib.call("g4q_decode_plan_create_ex", arr, pro, len(phases), max_tokens, rank, n_ranks,
                      ctypes.byref(self._h))
            if n_ranks > 1:
                self._connect(rank, n_ranks, group)
        elif n_ranks == 1:
            _lib.call("g4q_decode_plan_create", arr, len(phases), max_tokens, ctypes.byref(self._h))
        else:
            _lib.call("g4q_decode_plan_create_tp", arr, len(phases), max_tokens, rank, n_ranks, ctypes.byref(self._h))
            self._connect(rank, n_ranks, group)
        self.max_tokens = max_tokens

    def _connect(self, rank: int, n_ranks: int, group):
        """Exchange the plan's slot / key buffers with the other ranks (CUDA IPC handles over ``group``)."""
        slots, xkeys = ctypes.c_void_p(), ctypes.c_void_p()
        sb, kb = ctypes.c_uint64(), ctypes.c_uint64()
        _lib.call("g4q_decode_plan_buffers", self._h, ctypes.byref(slots), ctypes.byref(sb), ctypes.byref(xkeys),
                  ctypes.byref(kb))
        mine = []
        for ptr in (slots, xkeys):
            h = (ctypes.c_uint8 * _lib.IPC_HANDLE_BYTES)()
            _lib.call("g4q_ipc_handle", ptr, h)
            mine.append(bytes(h))
        allh = [None] * n_ranks
        torch.distributed.all_gather_object(allh, mine, group=group)
        peer_slots = (ctypes.c_void_p * n_ranks)()
        peer_keys = (ctypes.c_void_p * n_ranks)()
        for r in range(n_ranks):
            if r == rank:
                peer_slots[r], peer_keys[r] = slots.value, xkeys.value
                continue
            for j, dst in enumerate((peer_slots, peer_keys)):
                h = (ctypes.c_uint8 * _lib.IPC_HANDLE_BYTES).from_buffer_copy(allh[r][j])
                p = ctypes.c_void_p()
                _lib.call("g4q_ipc_open", h, ctypes.byref(p))
                self._opened.append(p)
                dst[r] = p.value
        _lib.call("g4q_decode_plan_set_peers", self._h, peer_slots, peer_keys)

    def run(self, M: int, *, eps: float = 1e-6, softcap: float = 30.0, row_offset: int = 0, tokens=None,
            values=None, keys=None, logits=None):
        ld = 0 if logits is None else logits.stride(0)
        _lib.call("g4q_decode_plan_run", self._h, M, eps, softcap, row_offset, _ptr(tokens), _ptr(values), _ptr(keys),
                  _ptr(logits), ld, _stream())

    def trace(self, enable: bool = True) -> Optional[torch.Tensor]:
        """Per-phase timeline of the following runs (profiling aid): returns the int64 device buffer
        [CTAs, phases, 19] of globaltimer stamps (ns) the tracing build of the kernel fills (entry,
        x's producers done, x staged, then each of the 16 warps' end of units), or None after
        switching back to the regular build."""
        words = ctypes.c_int64(0)
        _lib.call("g4q_decode_plan_trace", self._h, None, ctypes.byref(words))
        if not enable:
            self._trace = None
            return None
        buf = torch.zeros(words.value, dtype=torch.int64, device="cuda")
        _lib.call("g4q_decode_plan_trace", self._h, _ptr(buf), ctypes.byref(words))
        self._trace = buf
        return buf

    def free(self):
        for p in getattr(self, "_opened", []):
            _lib.call("g4q_ipc_close", p)
        self._opened = []
        if self._h:
            _lib.call("g4q_decode_plan_free", self._h)
            self._h = ctypes.c_void_p()
        self._keep = []

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


def synth_matrix(seed: int, rows: int, cols: int, bits: int = 4, group_size: int = 64, device=None):
    """Seeded synthetic MLX-layout matrix generated on the GPU (same values as the CPU oracle)."""
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    w = torch.empty((rows, cols * bits // 32), dtype=torch.uint32, device=dev)
    s = torch.empty((rows, cols // group_size), dtype=torch.bfloat16, device=dev)
    b = torch.empty_like(s)
    _lib.call("g4q_synth_matrix", seed & (2 ** 64 - 1), rows, cols, bits, group_size, _ptr(w), _ptr(s), _ptr(b),
              _stream())
    return w, s, b


def synth_normal(seed: int, shape, device=None) -> torch.Tensor:
    """Seeded bf16 ~ N(0, 1) tensor generated on the GPU (same values as the CPU oracle)."""
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    out = torch.empty(shape, dtype=torch.bfloat16, device=dev)
    _lib.call("g4q_synth_normal_bf16", seed & (2 ** 64 - 1), out.numel(), _ptr(out), _stream())
    return out
