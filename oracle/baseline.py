"""CPU baselines of the benchmark configurations (test / benchmark infrastructure only).

The reference runs these paths torch-eager on the host when no GPU kernel is bound
(its SDPA attention branch and fp32 modules).  The reference tree is not importable on
the GPU box, so each path is restated here in torch fp32 with the reference's own
structure and timed on all host cores; tests/test_oracle_golden.py pins the block
composition these restatements share (QKV -> per-head RMSNorm -> RoPE -> SDPA -> O)
to golden outputs of the reference's JointAttention.

  sdpa_cpu             config 2: F.scaled_dot_product_attention(q, k, v), fp32 -- the
                       SDPA branch of src/models/flux/attn.py:42-43 -- at the benchmark's
                       B x H x S x D (4 * B * H * S^2 * D FLOPs)
  joint_attention_cpu  config 1: JointAttention.forward (src/models/common/attn.py:190-236),
                       fp32, B=1, S=1024, dim 3072 = 24 x 128 heads, RMSNorm eps 1e-6 on
                       q/k, 2-D axial RoPE (theta 10000) over a 32 x 32 grid
  blocktopk_cpu        config 3: the block top-k form (pooling, fp32 block scores, top-k,
                       exact softmax over the kept 128-token key blocks), B=1, H=24,
                       S=16384, keep 16 of 128 blocks
  lumina_block_cpu     config 4: one JointTransformerBlock of the Lumina 2B shape
                       (src/models/lumina/image_two/model.py:31-102), 4352 tokens, 24/8
                       heads of 96, SwiGLU 6144; the step time is extrapolated by FLOPs
  flux_blocks_cpu      config 5: one double-stream and one single-stream Flux block
                       (src/models/flux/mmdit.py:62-231) at 4608 tokens; the step time is
                       19 x double + 38 x single (an extrapolation)
"""
from __future__ import annotations

import math
import os
import time
from contextlib import contextmanager

import torch
import torch.nn.functional as F


def attention_flops(B: int, H: int, Sq: int, Skv: int, D: int) -> float:
    return 4.0 * B * H * Sq * Skv * D


@contextmanager
def host_threads(threads: int | None = None):
    prev = torch.get_num_threads()
    torch.set_num_threads(threads or os.cpu_count() or 1)
    try:
        yield torch.get_num_threads()
    finally:
        torch.set_num_threads(prev)


def _timed(fn, reps: int = 1) -> float:
    best = float("inf")
    for _ in range(reps):
        t0 = time.perf_counter()
        fn()
        best = min(best, time.perf_counter() - t0)
    return best


def sdpa_cpu(B: int = 2, H: int = 24, S: int = 4608, D: int = 128, seed: int = 0, threads: int | None = None):
    """One call of the reference SDPA branch on the full B x H x S x D problem, fp32.
    Returns (seconds, flops, threads_used)."""
    with host_threads(threads) as thr, torch.inference_mode():
        g = torch.Generator().manual_seed(seed)
        q = torch.randn(B, H, S, D, generator=g)
        k = torch.randn(B, H, S, D, generator=g) + 3.0 * torch.randn(1, H, 1, D, generator=g)
        v = torch.randn(B, H, S, D, generator=g)
        dt = _timed(lambda: F.scaled_dot_product_attention(q, k, v))
        return dt, attention_flops(B, H, S, S, D), thr


def sdpa_cpu_sample(heads: int = 4, S: int = 4608, D: int = 128, seed: int = 0, threads: int | None = None):
    """The same on `heads` heads of one sequence."""
    return sdpa_cpu(1, heads, S, D, seed, threads)


# ------------------------------------------------------------ shared pieces --
def _linear(i: int, o: int, g: torch.Generator, bias: bool = False):
    """nn.Linear's default init range (uniform +-1/sqrt(in)), fp32."""
    b = 1.0 / math.sqrt(i)
    w = (torch.rand(o, i, generator=g) * 2 - 1) * b
    return w, ((torch.rand(o, generator=g) * 2 - 1) * b if bias else None)


def _rms(x, w, eps):
    return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * w


def _rope(x, f):
    """x [B, L, H, D] rotated by complex f [B, L, D/2] (src/kernels/__init__.py:126-142)."""
    xc = torch.view_as_complex(x.float().reshape(*x.shape[:-1], -1, 2))
    return torch.view_as_real(xc * f[:, :, None]).flatten(3)


def _axes_freqs(ids: torch.Tensor, axes, theta: float = 10000.0) -> torch.Tensor:
    """Multi-axis RoPE factors: ids [B, L, n_axes] -> complex64 [B, L, sum(axes) / 2]."""
    out = []
    for a, d in enumerate(axes):
        inv = 1.0 / theta ** (torch.arange(0, d, 2, dtype=torch.float64) / d)
        ang = ids[..., a].double()[..., None] * inv
        out.append(torch.polar(torch.ones_like(ang), ang))
    return torch.cat(out, -1).to(torch.complex64)


def _grid_ids(L_txt: int, h: int, w: int) -> torch.Tensor:
    ids = torch.zeros(1, L_txt + h * w, 3)
    ids[0, L_txt:, 1] = torch.arange(h).repeat_interleave(w)
    ids[0, L_txt:, 2] = torch.arange(w).repeat(h)
    return ids


def _attn(q, k, v, scale):
    """[B, L, H, D] SDPA with GQA (the reference's SDPA branch)."""
    rep = q.shape[2] // k.shape[2]
    if rep > 1:
        k, v = k.repeat_interleave(rep, 2), v.repeat_interleave(rep, 2)
    o = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2), scale=scale)
    return o.transpose(1, 2)


# ------------------------------------------------------------------ config 1 --
def joint_attention_cpu(seq: int = 1024, dim: int = 3072, heads: int = 24, reps: int = 3, threads=None):
    """Returns (seconds, flops, threads_used)."""
    hd = dim // heads
    with host_threads(threads) as thr, torch.inference_mode():
        g = torch.Generator().manual_seed(0)
        wq, wk, wv, wo = (_linear(dim, dim, g)[0] for _ in range(4))
        qn, kn = torch.ones(hd), torch.ones(hd)
        x = torch.randn(1, seq, dim, generator=g)
        side = int(round(math.sqrt(seq)))
        f = _axes_freqs(_grid_ids(0, side, seq // side), (hd - 2 * (hd // 4), hd // 4, hd // 4))

        def fwd():
            q = (x @ wq.T).view(1, seq, heads, hd)
            k = (x @ wk.T).view(1, seq, heads, hd)
            v = (x @ wv.T).view(1, seq, heads, hd)
            q, k = _rope(_rms(q, qn, 1e-6), f), _rope(_rms(k, kn, 1e-6), f)
            return _attn(q, k, v, 1.0 / math.sqrt(hd)).flatten(2) @ wo.T

        fwd()
        dt = _timed(fwd, reps)
        return dt, 4 * 2.0 * seq * dim * dim + attention_flops(1, heads, seq, seq, hd), thr


# ------------------------------------------------------------------ config 3 --
def blocktopk_cpu(S: int = 16384, H: int = 24, D: int = 128, keep: int = 16, threads=None):
    """Block pooling, fp32 block scores, top-k and exact attention over the kept blocks,
    batched torch fp32.  Returns (seconds, kept-attention flops, threads_used)."""
    nb = S // 128
    with host_threads(threads) as thr, torch.inference_mode():
        g = torch.Generator().manual_seed(0)
        q = torch.randn(H, S, D, generator=g)
        k = torch.randn(H, S, D, generator=g)
        v = torch.randn(H, S, D, generator=g)

        def fwd():
            pq = q.view(H, nb, 128, D).mean(2)
            pk = k.view(H, nb, 128, D).mean(2)
            idx = torch.topk(pq @ pk.transpose(1, 2), keep, dim=-1).indices.sort(-1).values   # [H, nb, keep]
            out = torch.empty_like(q)
            for h in range(H):   # one head at a time keeps the gathered blocks at ~130 MB
                ks = k[h].view(nb, 128, D)[idx[h]].reshape(nb, keep * 128, D)
                vs = v[h].view(nb, 128, D)[idx[h]].reshape(nb, keep * 128, D)
                s = q[h].view(nb, 128, D) @ ks.transpose(-1, -2) / math.sqrt(D)
                out[h] = (torch.softmax(s, -1) @ vs).view(S, D)
            return out

        fwd()
        dt = _timed(fwd)
        return dt, 4.0 * H * S * (keep * 128) * D, thr


# ------------------------------------------------------------------ config 4 --
def lumina_block_cpu(L: int = 4352, dim: int = 2304, heads: int = 24, kv_heads: int = 8, ffn: int = 6144,
                     threads=None):
    """One modulated JointTransformerBlock (attention + SwiGLU, sandwich RMSNorms, tanh
    gates).  Returns (seconds, flops of the block, threads_used)."""
    hd = dim // heads
    with host_threads(threads) as thr, torch.inference_mode():
        g = torch.Generator().manual_seed(0)
        wqkv = _linear(dim, (heads + 2 * kv_heads) * hd, g)[0]
        wo = _linear(heads * hd, dim, g)[0]
        w1, w3 = _linear(dim, ffn, g)[0], _linear(dim, ffn, g)[0]
        w2 = _linear(ffn, dim, g)[0]
        n = torch.ones(dim)
        x = torch.randn(1, L, dim, generator=g)
        mod = torch.randn(1, 4 * dim, generator=g) * 0.1
        f = _axes_freqs(_grid_ids(256, 64, (L - 256) // 64), (32, 32, 32))

        def fwd():
            s1, g1, s2, g2 = (c[:, None] for c in mod.chunk(4, -1))
            h = _rms(x, n, 1e-5) * (1 + s1)
            qkv = h @ wqkv.T
            q = qkv[..., :heads * hd].view(1, L, heads, hd)
            k = qkv[..., heads * hd:(heads + kv_heads) * hd].view(1, L, kv_heads, hd)
            v = qkv[..., (heads + kv_heads) * hd:].view(1, L, kv_heads, hd)
            q, k = _rope(_rms(q, torch.ones(hd), 1e-6), f), _rope(_rms(k, torch.ones(hd), 1e-6), f)
            y = x + torch.tanh(g1) * _rms(_attn(q, k, v, 1 / math.sqrt(hd)).flatten(2) @ wo.T, n, 1e-5)
            h = _rms(y, n, 1e-5) * (1 + s2)
            return y + torch.tanh(g2) * _rms((F.silu(h @ w1.T) * (h @ w3.T)) @ w2.T, n, 1e-5)

        fwd()
        dt = _timed(fwd)
        fl = 2.0 * L * dim * ((heads + 2 * kv_heads) * hd + heads * hd + 3 * ffn) + attention_flops(1, heads, L, L, hd)
        return dt, fl, thr


# ------------------------------------------------------------------ config 5 --
def flux_blocks_cpu(L_txt: int = 512, side: int = 64, dim: int = 3072, heads: int = 24, mlp_ratio: float = 4.0,
                    threads=None):
    """One double-stream and one single-stream Flux block at L_txt + side^2 tokens, fp32.
    Returns (seconds_double, seconds_single, threads_used)."""
    hd = dim // heads
    mlp = int(dim * mlp_ratio)
    L_img = side * side
    L = L_txt + L_img
    with host_threads(threads) as thr, torch.inference_mode():
        g = torch.Generator().manual_seed(0)
        f = _axes_freqs(_grid_ids(L_txt, side, side), (16, 56, 56))
        vec = torch.randn(1, dim, generator=g)
        one = torch.ones(hd)

        def stream(n_tok):
            return dict(mod=_linear(dim, 6 * dim, g, True), qkv=_linear(dim, 3 * dim, g, True),
                        proj=_linear(dim, dim, g, True), m0=_linear(dim, mlp, g, True),
                        m2=_linear(mlp, dim, g, True), x=torch.randn(1, n_tok, dim, generator=g))

        img, txt = stream(L_img), stream(L_txt)
        lin = lambda t, wb: F.linear(t, wb[0], wb[1])  # noqa: E731
        ln = lambda t: F.layer_norm(t, (dim,), eps=1e-6)  # noqa: E731

        def double():
            outs = []
            for s in (txt, img):
                m = lin(F.silu(vec), s["mod"]).chunk(6, -1)
                h = ln(s["x"]) * (1 + m[1][:, None]) + m[0][:, None]
                outs.append((m, lin(h, s["qkv"]).view(1, -1, 3, heads, hd)))
            q = torch.cat([o[1][:, :, 0] for o in outs], 1)
            k = torch.cat([o[1][:, :, 1] for o in outs], 1)
            v = torch.cat([o[1][:, :, 2] for o in outs], 1)
            q, k = _rope(_rms(q, one, 1e-6), f), _rope(_rms(k, one, 1e-6), f)
            a = _attn(q, k, v, 1 / math.sqrt(hd)).flatten(2)
            res = []
            for (m, _), s, sl in zip(outs, (txt, img), (slice(0, L_txt), slice(L_txt, L))):
                x = s["x"] + m[2][:, None] * lin(a[:, sl], s["proj"])
                h = ln(x) * (1 + m[4][:, None]) + m[3][:, None]
                res.append(x + m[5][:, None] * lin(F.gelu(lin(h, s["m0"]), approximate="tanh"), s["m2"]))
            return res

        smod = _linear(dim, 3 * dim, g, True)
        l1 = _linear(dim, 3 * dim + mlp, g, True)
        l2 = _linear(dim + mlp, dim, g, True)
        xs = torch.randn(1, L, dim, generator=g)

        def single():
            m = lin(F.silu(vec), smod).chunk(3, -1)
            h = ln(xs) * (1 + m[1][:, None]) + m[0][:, None]
            qkv, mlp_in = lin(h, l1).split([3 * dim, mlp], -1)
            qkv = qkv.view(1, L, 3, heads, hd)
            q, k = _rope(_rms(qkv[:, :, 0], one, 1e-6), f), _rope(_rms(qkv[:, :, 1], one, 1e-6), f)
            a = _attn(q, k, qkv[:, :, 2], 1 / math.sqrt(hd)).flatten(2)
            return xs + m[2][:, None] * lin(torch.cat([a, F.gelu(mlp_in, approximate="tanh")], -1), l2)

        double()
        td = _timed(double)
        single()
        ts = _timed(single)
        return td, ts, thr
