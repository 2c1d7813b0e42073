"""Helpers shared by the GPU parity tests (tensor <-> numpy bit views, tolerance checks)."""
import numpy as np
import torch


def u16(t: torch.Tensor) -> np.ndarray:
    return t.detach().contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def u32(t: torch.Tensor) -> np.ndarray:
    return t.detach().contiguous().view(torch.int32).cpu().numpy().view(np.uint32)


def dev_u16(a: np.ndarray, device, dtype=torch.bfloat16) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).to(device).view(dtype)


def dev_u32(a: np.ndarray, device) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int32)).to(device).view(torch.uint32)


def bf16_half_ulp(v: np.ndarray) -> np.ndarray:
    a = np.abs(v).astype(np.float64)
    e = np.floor(np.log2(np.maximum(a, 2.0 ** -126)))
    return 0.5 * 2.0 ** (e - 7)


def qmm_error(y_gpu: np.ndarray, y_exact: np.ndarray, bf16_out: bool):
    """(excess, rms): the largest |y_gpu - y_exact| beyond the bf16 output rounding (when the
    output is bf16), and rms(y_exact). The contract is excess <= 1e-2 * rms."""
    rms = float(np.sqrt(np.mean(y_exact.astype(np.float64) ** 2)))
    d = np.abs(y_gpu.astype(np.float64) - y_exact)
    if bf16_out:
        d = d - bf16_half_ulp(y_exact)
    return float(d.max()), rms


def assert_qmm_close(y_gpu: np.ndarray, y_exact: np.ndarray, bf16_out: bool, tol: float = 1e-2):
    excess, rms = qmm_error(y_gpu, y_exact, bf16_out)
    assert excess <= tol * rms, f"max excess |dy| = {excess:.3e} > {tol} * rms ({rms:.3e})"
