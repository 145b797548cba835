"""Restatements of the reference's elementwise / row kernels (test infrastructure only).

Each function follows the reference's eager body line for line in float32 numpy:
  rope_apply       src/kernels/__init__.py:126-142  (Triton: src/kernels/triton/rope.py:20-80)
  rmsnorm_apply    src/kernels/__init__.py:73-80    (Triton: src/kernels/triton/rmsnorm.py:22-69)
  inplace_softmax  src/kernels/__init__.py:83-87    (Triton: src/kernels/triton/softmax.py:22-79)
Pinned against tests/golden/ref_ops.npz, produced by the reference code itself.
"""
from __future__ import annotations

import numpy as np

from .numerics import round_to, round_f16


def rope_apply(xq: np.ndarray, xk: np.ndarray, freqs: np.ndarray, dtype: str = "f32", fp16_trig: bool = False):
    """xq [B,S,H,D], xk [B,S,Hk,D] (float32 values of `dtype`), freqs complex64 [B,S,D/2].

    Pair p of the last dim is the complex number x[2p] + i x[2p+1], multiplied by
    freqs[b, s, p] (kernels/__init__.py:128-140); every product is rounded to fp32
    separately, then the result is rounded to `dtype` (type_as, :142).  With
    fp16_trig the cos/sin are first rounded to fp16 as rope_triton does (rope.py:91-92).
    """
    c = np.real(freqs).astype(np.float32)
    s = np.imag(freqs).astype(np.float32)
    if fp16_trig:
        c, s = round_f16(c), round_f16(s)
    c = c[:, :, None, :]
    s = s[:, :, None, :]

    def rot(x):
        x = np.asarray(x, dtype=np.float32)
        x0 = x[..., 0::2]
        x1 = x[..., 1::2]
        re = (x0 * c).astype(np.float32) - (x1 * s).astype(np.float32)
        im = (x0 * s).astype(np.float32) + (x1 * c).astype(np.float32)
        out = np.empty_like(x)
        out[..., 0::2] = re
        out[..., 1::2] = im
        return round_to(out, dtype)

    return rot(xq), (rot(xk) if xk is not None else None)


def rmsnorm_apply(x: np.ndarray, w: np.ndarray, eps: float, x_dtype: str = "f32", out_dtype: str | None = None,
                  fused: bool = False) -> np.ndarray:
    """x [..., N] float32 values of x_dtype, w [N].

    eager (kernels/__init__.py:74-80): n = x * rsqrt(mean(x^2) + eps) in fp32,
    rounded to x's dtype (type_as), then * w, rounded to the promoted dtype.
    fused (src/kernels/triton/rmsnorm.py:62-68): (x * rsqrt) * w in fp32, one rounding at the end.
    """
    out_dtype = out_dtype or x_dtype
    x = np.asarray(x, dtype=np.float32)
    w = np.asarray(w, dtype=np.float32)
    ms = (np.sum(x.astype(np.float64) ** 2, axis=-1, keepdims=True) / x.shape[-1]).astype(np.float32)
    r = (np.float32(1.0) / np.sqrt((ms + np.float32(eps)).astype(np.float64))).astype(np.float32)
    n = (x * r).astype(np.float32)
    if not fused:
        n = round_to(n, x_dtype)
    return round_to((n * w).astype(np.float32), out_dtype)


def softmax_lastdim(x: np.ndarray, dtype: str = "f32") -> np.ndarray:
    """Row softmax over the last dim in fp32 (torch.softmax, kernels/__init__.py:87)."""
    x = np.asarray(x, dtype=np.float64)
    m = np.max(x, axis=-1, keepdims=True)
    e = np.exp(x - m)
    return round_to((e / np.sum(e, axis=-1, keepdims=True)).astype(np.float32), dtype)


def rope_scatter(x: np.ndarray, f: np.ndarray, idx: np.ndarray, y: np.ndarray) -> np.ndarray:
    """RAS RoPE with row scatter (src/kernels/cuda/ras.cu:12-52) with the stated rounding:
    x [B, N, H, D] (bf16 values as float32), f [N, D] float32 (cos, sin per pair), idx [N],
    y [B, M, H, D] updated copy.  Per pair: re = x0 f0 - x1 f1, im = x0 f1 + x1 f0, every
    product and sum rounded to fp32, then to bf16."""
    x = np.asarray(x, np.float32)
    y = np.array(y, np.float32, copy=True)
    a0, a1 = x[..., 0::2], x[..., 1::2]
    c = np.asarray(f, np.float32)[None, :, None, 0::2]
    s = np.asarray(f, np.float32)[None, :, None, 1::2]
    re = (a0 * c).astype(np.float32) - (a1 * s).astype(np.float32)
    im = (a0 * s).astype(np.float32) + (a1 * c).astype(np.float32)
    out = np.empty_like(x)
    out[..., 0::2] = re.astype(np.float32)
    out[..., 1::2] = im.astype(np.float32)
    y[:, np.asarray(idx)] = round_to(out, "bf16")
    return y


def partially_linear(x: np.ndarray, w: np.ndarray, idx: np.ndarray, out: np.ndarray) -> np.ndarray:
    """RAS row-indexed linear (src/kernels/triton/ras.py:28-128): out[b, idx[m]] = x[b, m] . w^T
    (float64 here; the device accumulates in fp32 and rounds once to the output dtype)."""
    out = np.array(out, np.float64, copy=True)
    out[:, np.asarray(idx)] = np.einsum("bmk,nk->bmn", np.asarray(x, np.float64), np.asarray(w, np.float64))
    return out
