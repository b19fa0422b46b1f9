"""Helpers for the GPU parity tests (conversion between the golden bit
patterns, numpy and torch)."""
import numpy as np
import torch

DT_TORCH = {0: torch.float32, 1: torch.bfloat16, 2: torch.float16}


def from_bits(a: np.ndarray, dt: int) -> torch.Tensor:
    """Golden array (bf16/f16 as uint16) -> torch tensor of dtype code dt."""
    if dt == 0:
        return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32))
    t = torch.from_numpy(np.ascontiguousarray(a).astype(np.uint16).view(np.int16))
    return t.view(DT_TORCH[dt])


def to_bits(t: torch.Tensor) -> np.ndarray:
    t = t.detach().contiguous().cpu()
    if t.dtype in (torch.bfloat16, torch.float16):
        return t.view(torch.int16).numpy().view(np.uint16).copy()
    if t.dtype == torch.float8_e4m3fnuz:
        return t.view(torch.uint8).numpy().copy()
    return t.numpy().copy()


def to_f32(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().cpu().numpy()


def same_float_bits(a: np.ndarray, b: np.ndarray, dt: int) -> bool:
    """Bitwise equality, NaN == NaN (payloads are not part of the format)."""
    from oracle import oracle as orc
    fa = orc.to_f32(a.reshape(-1), dt)
    fb = orc.to_f32(b.reshape(-1), dt)
    na, nb = np.isnan(fa), np.isnan(fb)
    if not np.array_equal(na, nb):
        return False
    return np.array_equal(fa[~na].view(np.uint32), fb[~nb].view(np.uint32))
