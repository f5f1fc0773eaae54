"""bf16 rounding emulation for the oracle (round-to-nearest-even of fp32)."""
from __future__ import annotations

import numpy as np


def bf16_round(x) -> np.ndarray:
    """Rounds float32 values to the nearest bfloat16 (ties to even), kept as float32."""
    x = np.asarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    lsb = (u >> np.uint64(16)) & np.uint64(1)
    r = ((u + np.uint64(0x7FFF) + lsb) & np.uint64(0xFFFF0000)).astype(np.uint32).view(np.float32)
    return np.where(np.isnan(x), x, r).astype(np.float32)


def bf16_bits(x) -> np.ndarray:
    """uint16 bit patterns of bf16-rounded values."""
    return (bf16_round(x).view(np.uint32) >> np.uint32(16)).astype(np.uint16)


def from_bf16_bits(b) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << np.uint32(16)).view(np.float32)
