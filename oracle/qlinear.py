"""Quantized linears restated on the CPU (test infrastructure only).

The reference quantizes nn.Linear weights through torchao 0.7.0 (src/quant.py:209-241;
version pinned only in get-lumina.bat:2, package absent here), after casting the model
to the qdtype's activation dtype (fp16 for qint8 / qfloat8, src/quant.py:326,331,383).
`quantize_weight_torchao` restates the steps of torchao 0.7.0's choose_qparams_affine and
quantize_affine (torchao/quantization/quant_primitives.py) as the reference configures
them -- symmetric, one block per output row (block_size=(1, in)), eps = fp32 epsilon,
scale_dtype left to default to the weight's dtype T -- with each tensor op rounded to T
as the library computes it (fp32 opmath, result rounded to T):
  amax  = max(-min(min_row, 0), max(max_row, 0))
  scale = clamp(T(amax / ((qmax - qmin) / 2)), min=eps)  -- 127.5 for int8, 448 for e4m3
  int8:  code = clamp(round(T(w * T(1.0 / scale))) + 0, -128, 127).to(int8)
  e4m3:  code = clamp(T(w * T(scale.reciprocal())), -448, 448).to(float8_e4m3fn)
PARITY UNPINNED against torchao itself (not installed, no golden vectors in the
reference); the CUDA weight quantizer is checked bit-exactly against this restatement.

The W8A8 activation quantizer (per token, no counterpart in the reference) uses fp32:
  int8:  amax = max|row| (fp32); scale = max(amax / 127.5, FLT_EPSILON); code = rint(x / scale)
         clamped to [-128, 127].
  e4m3:  scale = amax / 448 (1.0 for a zero row); code = e4m3(x * (448 / amax)) with
         round-to-nearest-even, saturating.
Linear outputs (float) are compared within tolerance:
  weight-only:  y = (x . codes^T) * scale[n] + bias       (fp32 accumulation)
  W8A8 e4m3:    y = (e4m3(x) . codes^T) * sx[m] * sw[n] + bias
"""
from __future__ import annotations

import numpy as np

from .numerics import e4m3_bits_to_f32, round_to, to_e4m3_bits

FLT_EPS = np.float32(np.finfo(np.float32).eps)


def quantize_weight_torchao(w: np.ndarray, fmt: str, dtype: str = "f16"):
    """w [N, K] (float32 values of `dtype`: "f16", "bf16" or "f32") -> (codes, fp32 scales):
    int8 codes, or uint8 e4m3 bit patterns for fmt "e4m3"."""
    w = round_to(np.asarray(w, dtype=np.float32), dtype)
    lo = np.minimum(w.min(axis=1), np.float32(0))
    hi = np.maximum(w.max(axis=1), np.float32(0))
    amax = np.maximum(-lo, hi).astype(np.float32)
    den = np.float32(127.5 if fmt == "int8" else 448.0)
    scale = np.maximum(round_to((amax / den).astype(np.float32), dtype), FLT_EPS).astype(np.float32)
    with np.errstate(divide="ignore", over="ignore", invalid="ignore"):
        recip = round_to((np.float32(1.0) / scale).astype(np.float32), dtype)
        y = round_to((w * recip[:, None]).astype(np.float32), dtype)
    if fmt == "int8":
        c = np.clip(np.rint(y), -128, 127)
        return np.where(np.isnan(y), 0, c).astype(np.int8), scale
    # 0 * inf (a row whose reciprocal scale overflowed) is the positive canonical NaN on the
    # GPU, where the reference quantizes; the host's default NaN can carry the sign bit
    y = np.where(np.isnan(y), np.float32(np.nan), y).astype(np.float32)
    return to_e4m3_bits(y), scale


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
