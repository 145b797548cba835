"""Quantized linears restated on the CPU (test infrastructure only).

The reference quantizes nn.Linear weights through torchao 0.7.0 (src/quant.py:209-241;
version pinned only in get-lumina.bat:2, package absent here): symmetric int8 with
one scale per output row (block_size=(1, in), eps = fp32 epsilon) and float8 e4m3
with one scale per output row.  PARITY UNPINNED against torchao itself (not
installed, no golden vectors in the reference); the rules below are this build's
stated definitions, checked bit-exactly against the CUDA quantizers:
  int8:  amax = max|row| (fp32); scale = max(amax / 127.5, FLT_EPSILON) (the symmetric
         mapping's (qmax - qmin) / 2 denominator); code = rint(x / scale) clamped
         to [-128, 127].
  e4m3:  scale = amax / 448 (1.0 for a zero row); code = e4m3(x * (448 / amax)) with
         round-to-nearest-even, saturating.
Linear outputs (float) are compared within tolerance:
  weight-only:  y = (x . codes^T) * scale[n] + bias       (fp32 accumulation)
  W8A8 e4m3:    y = (e4m3(x) . codes^T) * sx[m] * sw[n] + bias
"""
from __future__ import annotations

import numpy as np

from .numerics import e4m3_bits_to_f32, to_e4m3_bits

FLT_EPS = np.float32(np.finfo(np.float32).eps)


def quantize_rows_int8(x: np.ndarray):
    x = np.asarray(x, dtype=np.float32)
    am = np.max(np.abs(x), axis=1).astype(np.float32)
    scale = np.maximum((am / np.float32(127.5)).astype(np.float32), FLT_EPS).astype(np.float32)
    codes = np.clip(np.rint((x / scale[:, None]).astype(np.float32)), -128, 127).astype(np.int8)
    return codes, scale


def quantize_rows_e4m3(x: np.ndarray):
    x = np.asarray(x, dtype=np.float32)
    am = np.max(np.abs(x), axis=1).astype(np.float32)
    safe = np.where(am > 0, am, np.float32(1.0)).astype(np.float32)
    scale = np.where(am > 0, (safe / np.float32(448.0)).astype(np.float32), np.float32(1.0)).astype(np.float32)
    inv = np.where(am > 0, (np.float32(448.0) / safe).astype(np.float32), np.float32(1.0)).astype(np.float32)
    codes = to_e4m3_bits((x * inv[:, None]).astype(np.float32))
    return codes, scale


def linear_weight_only(x, codes, scale, bias=None, fp8=False):
    w = e4m3_bits_to_f32(codes) if fp8 else np.asarray(codes, dtype=np.float32)
    y = (np.asarray(x, np.float64) @ w.astype(np.float64).T) * np.asarray(scale, np.float64)[None, :]
    if bias is not None:
        y = y + np.asarray(bias, np.float64)[None, :]
    return y.astype(np.float32)


def linear_w8a8_e4m3(x, codes, scale, bias=None):
    xc, xs = quantize_rows_e4m3(x)
    y = (e4m3_bits_to_f32(xc).astype(np.float64) @ e4m3_bits_to_f32(codes).astype(np.float64).T)
    y = y * xs[:, None].astype(np.float64) * np.asarray(scale, np.float64)[None, :]
    if bias is not None:
        y = y + np.asarray(bias, np.float64)[None, :]
    return y.astype(np.float32)
