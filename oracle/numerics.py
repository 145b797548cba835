"""Bit-level helpers shared by the oracle restatements (test infrastructure only)."""
from __future__ import annotations

import numpy as np


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round float32 -> bfloat16 (nearest even), returned as uint16 bit patterns."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    nan = np.isnan(np.asarray(x, dtype=np.float32))
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = 0x7FC0
    return r


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def round_bf16(x: np.ndarray) -> np.ndarray:
    """float32 values rounded to the nearest bfloat16 (returned as float32)."""
    return bf16_bits_to_f32(f32_to_bf16_bits(x))


def round_f16(x: np.ndarray) -> np.ndarray:
    return np.asarray(x, dtype=np.float32).astype(np.float16).astype(np.float32)


def round_to(x: np.ndarray, dtype: str) -> np.ndarray:
    if dtype == "bf16":
        return round_bf16(x)
    if dtype == "f16":
        return round_f16(x)
    return np.asarray(x, dtype=np.float32)


def to_e4m3_bits(x: np.ndarray) -> np.ndarray:
    """float32 -> float8 e4m3fn bit patterns, round to nearest even, saturating at +-448."""
    import torch

    t = torch.from_numpy(np.clip(np.asarray(x, dtype=np.float32), -448.0, 448.0))
    return t.to(torch.float8_e4m3fn).view(torch.uint8).numpy()


def e4m3_bits_to_f32(b: np.ndarray) -> np.ndarray:
    import torch

    t = torch.from_numpy(np.ascontiguousarray(b, dtype=np.uint8)).view(torch.float8_e4m3fn)
    return t.to(torch.float32).numpy()
