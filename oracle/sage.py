"""SageAttention-style quantized attention, restated on the CPU (test infrastructure only).

The reference reaches this path through the third-party `sageattention` package:
    sageattn(q, k, v)                       src/models/flux/attn.py:39-41 (HND layout)
    sageattn_varlen(q, k, v, cu_seqlens...) src/models/common/attn.py:109-120
That package is not vendored, its version is not pinned anywhere in the reference
tree (and it is not installed here), and no test or golden vector of the reference touches it, so
parity of the quantization codes is UNPINNED against the package itself.  This module
restates the published SageAttention / SageAttention2 algorithm (Zhang et al.,
"SageAttention", ICLR 2025; "SageAttention2", 2025) with every rounding step stated
so that the CUDA path can be checked bit-exactly against it:

  1. K smoothing: km[c] = (float32)(sum_fp64(k[:, c]) / len) per (sequence, kv head);
     k' = float32(k) - km  (one fp32 rounding).
  2. Q pre-scale: q' = float32(q) * c with c = float32(float64(float32(sm_scale)) * log2(e)),
     which folds the softmax scale and the base-2 exponent into Q.
  3. INT8 per 64-token block (per sequence, head), the rule of the published SageAttention
     Triton quantizer (sageattention 1.0.x, `quant_per_block.py`, quant_per_block_int8_kernel:
     `scale = max|x| / 127.`, `x_int8 = x / scale`, `x_int8 += 0.5 * where(x_int8 >= 0, 1, -1)`,
     `x_int8.to(int8)`): scale = float32(amax / 127); t = float32(x / scale) (IEEE division;
     Triton may lower `/` to an approximate divide -- the correctly rounded quotient is the
     definition here so the CPU can reproduce it); u = float32(t + 0.5 * sign(t)) (+0.5 for
     t >= 0, -0.5 otherwise); code = trunc(u) toward zero, which never leaves [-127, 127].
     An all-zero block gets scale 1.0 and codes 0 (the Triton kernel divides 0 by 0 there).
     Block size 64 for Q and K is the benchmarked configuration's (the Triton v1 kernels
     use 128-token Q blocks).
  4. V per channel over the whole sequence: vinv = 448 / amax, vs = amax / 448 (fp32;
     1.0 if zero); v8 = e4m3(float32(v * vinv)) with round-to-nearest-even.
  5. Logits (base 2): S = (int32)(qcode . kcode) * (sq * sk)  (fp32 product of scales).
  6. Softmax in base 2; P = e4m3(448 * 2^(S - rowmax)); O = (P . v8) * vs / sum(448 * 2^(S - rowmax)).
     The GPU kernel does step 6 online (running max per 128-key tile), so its P
     codes are taken against the running max; outputs agree within a tolerance, not bitwise.
"""
from __future__ import annotations

import math

import numpy as np

from .numerics import e4m3_bits_to_f32, to_e4m3_bits

LOG2E = 1.4426950408889634
QBLOCK = 64


def q_prescale(sm_scale: float) -> np.float32:
    return np.float32(float(np.float32(sm_scale)) * LOG2E)


def block_codes(x: np.ndarray, scale: np.float32) -> np.ndarray:
    """Step 3's element rule for one block: x float32, scale float32 > 0 -> int8 codes."""
    t = (np.asarray(x, np.float32) / np.float32(scale)).astype(np.float32)
    u = (t + np.where(t >= 0, np.float32(0.5), np.float32(-0.5))).astype(np.float32)
    return np.trunc(u).astype(np.int8)


def _block_quant(x: np.ndarray):
    """x [S, D] float32 -> (codes int8 [S, D], scales float32 [ceil(S/64)])."""
    x = np.asarray(x, dtype=np.float32)
    S, D = x.shape
    nb = (S + QBLOCK - 1) // QBLOCK
    pad = np.zeros((nb * QBLOCK, D), np.float32)
    pad[:S] = x
    blk = pad.reshape(nb, QBLOCK, D)
    am = np.abs(blk).max(axis=(1, 2)).astype(np.float32) if nb else np.zeros(0, np.float32)
    scales = np.where(am > 0, (am / np.float32(127.0)).astype(np.float32), np.float32(1.0)).astype(np.float32)
    codes = block_codes(blk, scales[:, None, None]).reshape(nb * QBLOCK, D)[:S]
    return codes, scales


def quantize_q(q: np.ndarray, sm_scale: float):
    """Steps 2-3 for the query rows of one (sequence, head): (codes, scales)."""
    qx = (np.asarray(q, dtype=np.float32) * q_prescale(sm_scale)).astype(np.float32)
    return _block_quant(qx)


def quantize_kv(k: np.ndarray, v: np.ndarray):
    """Steps 1, 3 and 4 for one (sequence, kv head): dict with kcodes, kscales, kmean, v8, vscale."""
    k = np.asarray(k, dtype=np.float32)
    kmean = (np.sum(k.astype(np.float64), axis=0) / max(k.shape[0], 1)).astype(np.float32)
    kx = (k - kmean[None, :]).astype(np.float32)
    kcodes, kscales = _block_quant(kx)
    v = np.asarray(v, dtype=np.float32)
    am = np.max(np.abs(v), axis=0).astype(np.float32) if v.shape[0] else np.zeros(v.shape[1], np.float32)
    safe = np.where(am > 0, am, np.float32(1.0)).astype(np.float32)
    vscale = np.where(am > 0, (safe / np.float32(448.0)).astype(np.float32), np.float32(1.0)).astype(np.float32)
    vinv = np.where(am > 0, (np.float32(448.0) / safe).astype(np.float32), np.float32(1.0)).astype(np.float32)
    v8 = to_e4m3_bits((v * vinv[None, :]).astype(np.float32))
    return dict(kcodes=kcodes, kscales=kscales, kmean=kmean, v8=v8, vscale=vscale)


def quantize_head(q: np.ndarray, k: np.ndarray, v: np.ndarray, sm_scale: float):
    """One sequence, one (q head, kv head) pair.  q [Sq, D], k/v [Skv, D] float32 values.

    Returns dict with qcodes, qscales, kcodes, kscales, kmean, v8 (uint8 e4m3 bits), vscale.
    """
    qcodes, qscales = quantize_q(q, sm_scale)
    return dict(qcodes=qcodes, qscales=qscales, **quantize_kv(k, v))


def attention_from_codes(qz: dict, rows=None) -> np.ndarray:
    """Step 5-6 on the quantized codes of one head: returns O [Sq, D] float32 (only the
    query rows `rows`, in that order, when given)."""
    # integer dot products in float64 (exact: |sum| <= 128 * 127^2 < 2^53), through BLAS
    qc = qz["qcodes"].astype(np.float64)
    kc = qz["kcodes"].astype(np.float64)
    Sq, Skv = qc.shape[0], kc.shape[0]
    sq = np.repeat(qz["qscales"], QBLOCK)[:Sq]
    if rows is not None:
        qc, sq = qc[rows], sq[rows]
    s_int = qc @ kc.T
    sk = np.repeat(qz["kscales"], QBLOCK)[:Skv]
    sc = (sq[:, None] * sk[None, :]).astype(np.float32)
    logits = (s_int.astype(np.float32) * sc).astype(np.float32)
    m = np.max(logits, axis=1, keepdims=True)
    p448 = np.exp2((logits - m).astype(np.float64) + math.log2(448.0)).astype(np.float32)
    l = np.sum(p448.astype(np.float64), axis=1, keepdims=True)
    p8 = e4m3_bits_to_f32(to_e4m3_bits(p448))
    v8 = e4m3_bits_to_f32(qz["v8"])
    o = (p8.astype(np.float64) @ v8.astype(np.float64)) * qz["vscale"][None, :].astype(np.float64) / l
    return o.astype(np.float32)


def sageattn(q: np.ndarray, k: np.ndarray, v: np.ndarray, sm_scale: float | None = None) -> np.ndarray:
    """Dense HND: q [B, Hq, Sq, D], k/v [B, Hkv, Skv, D] -> O [B, Hq, Sq, D] (float32)."""
    B, Hq, Sq, D = q.shape
    Hkv = k.shape[1]
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(D)
    out = np.zeros((B, Hq, Sq, D), dtype=np.float32)
    for b in range(B):
        for h in range(Hq):
            hk = h // (Hq // Hkv)
            out[b, h] = attention_from_codes(quantize_head(q[b, h], k[b, hk], v[b, hk], sm_scale))
    return out


def sdpa_reference(q: np.ndarray, k: np.ndarray, v: np.ndarray, sm_scale: float | None = None) -> np.ndarray:
    """The reference's unquantized SDPA branch (src/models/common/attn.py:123-130,
    src/models/flux/attn.py:42-43) in float64 on the same inputs, HND layout, GQA."""
    B, Hq, Sq, D = q.shape
    Hkv = k.shape[1]
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(D)
    rep = Hq // Hkv
    kk = np.repeat(np.asarray(k, np.float64), rep, axis=1)
    vv = np.repeat(np.asarray(v, np.float64), rep, axis=1)
    s = np.einsum("bhqd,bhkd->bhqk", np.asarray(q, np.float64), kk) * sm_scale
    s -= s.max(axis=-1, keepdims=True)
    p = np.exp(s)
    p /= p.sum(axis=-1, keepdims=True)
    return np.einsum("bhqk,bhkd->bhqd", p, vv).astype(np.float32)


_UNSWZ = np.array([[r * 8 + (c ^ (r & 7)) for c in range(8)] for r in range(128)], dtype=np.int64).reshape(-1)


def unswizzle_tile(tile: np.ndarray) -> np.ndarray:
    """Inverse of the 128-byte swizzle used by the GPU tile layout: tile [..., 16384] uint8
    -> logical [..., 128 rows, 128 bytes].  Row r, 16-byte chunk c lives at r*128 + (c ^ (r & 7))*16."""
    t = np.asarray(tile, dtype=np.uint8)
    lead = t.shape[:-1]
    chunks = t.reshape(*lead, 1024, 16)
    return chunks[..., _UNSWZ, :].reshape(*lead, 128, 128)
