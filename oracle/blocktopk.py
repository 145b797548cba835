"""Top-k block-sparse attention, restated on the CPU (test infrastructure only).

The reference's sparse path is `topk_attn` (src/kernels/__init__.py:146-195): per-token
top-k over a dense [B, H, S, S] score matrix, the mask cached across layers in the
module global POS_DICT (src/models/common/attn.py:20, :24-56).  As written it is
numerically broken (matmuls written into their own aliased inputs at :173 and :192,
and the computed mask is never applied when POS_DICT is None, :179-188), and its
dense S x S scores do not fit at 16384 tokens, so it yields no usable golden vectors:
PARITY UNPINNED against the reference.  This module states the block form the GPU
path implements, with every rounding step fixed so block indices compare bit-exactly:

  1. Mean-pool Q and K over 128-token blocks per (batch, head): fp64 sum of the
     block's rows (exact for bf16/fp16 inputs) divided by the row count, rounded to fp32.
     A ragged last block averages its valid rows.
  2. Block scores: score[i, j] = sum_d float64(pq[i, d]) * float64(pk[j, d]), products
     and partial sums in fp64, d ascending, rounded once to fp32.
  3. Per query block keep `keep` key blocks: descending score, the lower block index
     wins ties; the kept indices are reported in ascending order (int32).
  4. Attention of every query row over the rows of its kept key blocks: exact softmax
     of q.k * sm_scale (keys beyond S masked), times V.
"""
from __future__ import annotations

import math

import numpy as np

BLOCK = 128


def pool_blocks(x: np.ndarray) -> np.ndarray:
    """x [S, D] -> [ceil(S/128), D] fp32 block means (step 1)."""
    S, D = x.shape
    nb = (S + BLOCK - 1) // BLOCK
    out = np.empty((nb, D), dtype=np.float32)
    x64 = np.asarray(x, dtype=np.float64)
    for i in range(nb):
        blk = x64[i * BLOCK:(i + 1) * BLOCK]
        out[i] = (blk.sum(axis=0) / blk.shape[0]).astype(np.float32)
    return out


def block_scores(pq: np.ndarray, pk: np.ndarray) -> np.ndarray:
    """[nq, D] x [nk, D] -> [nq, nk] fp32 with the fixed fp64 summation order of step 2."""
    a = np.asarray(pq, dtype=np.float64)
    b = np.asarray(pk, dtype=np.float64)
    acc = np.zeros((a.shape[0], b.shape[0]), dtype=np.float64)
    for d in range(a.shape[1]):
        acc = acc + np.outer(a[:, d], b[:, d])
    return acc.astype(np.float32)


def select(scores: np.ndarray, keep: int) -> np.ndarray:
    """[nq, nk] fp32 -> [nq, keep] int32, ascending block indices (step 3)."""
    nq, nk = scores.shape
    keep = min(keep, nk)
    out = np.empty((nq, keep), dtype=np.int32)
    idx = np.arange(nk)
    for i in range(nq):
        # stable sort on -score keeps the lower index first among equal scores
        order = np.argsort(-scores[i].astype(np.float64), kind="stable")
        out[i] = np.sort(idx[order[:keep]])
    return out


def select_head(q: np.ndarray, k: np.ndarray, keep: int) -> np.ndarray:
    """One (batch, head): q [S, D], k [S, D] -> kept block indices [nqb, keep]."""
    return select(block_scores(pool_blocks(q), pool_blocks(k)), keep)


def attention_head(q: np.ndarray, k: np.ndarray, v: np.ndarray, idx: np.ndarray, sm_scale: float) -> np.ndarray:
    """Step 4 for one head: q [Sq, D] holding the query blocks idx rows refer to (row i of
    idx = q rows i*128..), k/v [S, D], idx [nqb, keep] -> O [Sq, D] fp32 (fp64 math)."""
    Sq, D = q.shape
    S = k.shape[0]
    q64, k64, v64 = (np.asarray(t, dtype=np.float64) for t in (q, k, v))
    out = np.zeros((Sq, D), dtype=np.float32)
    for i in range(idx.shape[0]):
        rows = slice(i * BLOCK, min((i + 1) * BLOCK, Sq))
        cols = np.concatenate([np.arange(j * BLOCK, min((j + 1) * BLOCK, S)) for j in idx[i]])
        s = q64[rows] @ k64[cols].T * sm_scale
        s -= s.max(axis=1, keepdims=True)
        p = np.exp(s)
        p /= p.sum(axis=1, keepdims=True)
        out[rows] = (p @ v64[cols]).astype(np.float32)
    return out


def blocksparse_attention(q, k, v, keep: int, sm_scale: float | None = None):
    """HND: q [B, Hq, S, D], k/v [B, Hkv, S, D] -> (O [B, Hq, S, D], idx [B, Hq, nqb, keep])."""
    B, Hq, S, D = q.shape
    Hkv = k.shape[1]
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(D)
    nqb = (S + BLOCK - 1) // BLOCK
    keep = min(keep, nqb)
    out = np.zeros(q.shape, dtype=np.float32)
    idx = np.zeros((B, Hq, nqb, keep), dtype=np.int32)
    for b in range(B):
        for h in range(Hq):
            hk = h // (Hq // Hkv)
            idx[b, h] = select_head(q[b, h], k[b, hk], keep)
            out[b, h] = attention_head(q[b, h], k[b, hk], v[b, hk], idx[b, h], sm_scale)
    return out, idx


def make_hot_inputs(B, H, S, D, hot=4, boost=2.0, seed=0):
    """Seeded synthetic inputs of the block-sparse benchmark: Q, K, V ~ N(0, 1); every
    query block i gets a random unit direction u_i added to its rows (scaled by `boost`),
    and `hot` randomly chosen key blocks get boost * u_i added to their rows, so those
    key blocks score high for query block i ("query-aligned hot key blocks")."""
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((B, H, S, D), dtype=np.float32)
    k = rng.standard_normal((B, H, S, D), dtype=np.float32)
    v = rng.standard_normal((B, H, S, D), dtype=np.float32)
    nb = (S + BLOCK - 1) // BLOCK
    for b in range(B):
        for h in range(H):
            u = rng.standard_normal((nb, D))
            u /= np.linalg.norm(u, axis=1, keepdims=True)
            for i in range(nb):
                q[b, h, i * BLOCK:(i + 1) * BLOCK] += (boost * u[i]).astype(np.float32)
                for j in rng.choice(nb, size=min(hot, nb), replace=False):
                    k[b, h, j * BLOCK:(j + 1) * BLOCK] += (boost * u[i]).astype(np.float32)
    return q, k, v
