"""bf16 helpers on numpy arrays (test infrastructure; see oracle/__init__.py)."""

from __future__ import annotations

import numpy as np
import torch


def f32_to_bits(x: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 bit pattern (uint16), round to nearest even (finite inputs)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    bias = ((u >> 16) & 1) + np.uint32(0x7FFF)
    return ((u + bias) >> 16).astype(np.uint16)


def bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def bf16r(x: np.ndarray) -> np.ndarray:
    """Round fp32 values to bf16 and back (what a bf16 store then load does)."""
    return bits_to_f32(f32_to_bits(x))


def torch_to_bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def bits_to_torch(b: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(b, dtype=np.uint16).view(np.int16)).view(torch.bfloat16)
