"""Lumina-Image-2.0-shaped DiT forward built from the B200 ops.

Structure of src/models/lumina/image_two/model.py (LuminaDiT :154-414, JointTransformerBlock
:31-102) with JointAttention (src/models/common/attn.py:133-236) and the SwiGLU
LlamaFeedForward (src/models/common/nextdit.py:81-125); the 2B shape of
src/models/lumina/image_two/pipeline.py:25-37 (dim 2304, 26 layers, 2 + 2 refiner layers,
24 query / 8 KV heads of 96, RoPE axes (32, 32, 32)) with the SwiGLU hidden width a
parameter.  Weights are random; every linear is an INT8 weight-only QLinear (the qint8
path of src/quant.py:209-224, 323-327).

Per block (B*L rows, dim columns):
  qkv GEMM -> fused q/k RMSNorm + RoPE -> Sage attention at head_dim 96 (GQA 24/8) -> wo
  GEMM -> x += tanh(gate) * RMSNorm(.) and the next norm-modulate in one pass ->
  w1/w3 GEMM with the SwiGLU epilogue -> w2 GEMM -> the same fused residual pass producing
  the next block's input.

Batch parallelism: samples are independent, so on P GPUs each rank runs its own samples
with no collective (the B=8 over 8 GPUs configuration).
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F
from torch import nn

from .attention import sageattn
from .dit import rope_freqs
from .kernels import qkv_norm_rope, rms_gate_residual
from .quant import QLinear, gemm, glu_interleave, ln_modulate, quantize_rows


def _rand_weight(out_f: int, in_f: int, device, gen) -> torch.Tensor:
    bound = 1.0 / math.sqrt(in_f)
    return (torch.rand(out_f, in_f, device=device, generator=gen) * 2 - 1).mul_(bound).to(torch.bfloat16)


def _qlin(w: torch.Tensor, bias: torch.Tensor | None, mode: str) -> QLinear:
    codes, scale = quantize_rows(w, "int8" if mode == "int8" else "e4m3")
    return QLinear(codes, scale, bias, mode, w.shape[1], w.shape[0])


def _rand_qlin(in_f, out_f, mode, device, gen, bias=True) -> QLinear:
    w = _rand_weight(out_f, in_f, device, gen)
    b = None
    if bias:
        b = ((torch.rand(out_f, device=device, generator=gen) * 2 - 1) / math.sqrt(in_f)).to(torch.bfloat16)
    return _qlin(w, b, mode)


def pad_head_columns(w: torch.Tensor, heads: int, hd: int, hd_pad: int) -> torch.Tensor:
    """Output-projection weight [out, heads*hd] -> [out, heads*hd_pad] with zero columns on
    each head's padding, so the GEMM reads the padded attention output directly."""
    out_f = w.shape[0]
    p = torch.zeros(out_f, heads, hd_pad, dtype=w.dtype, device=w.device)
    p[:, :, :hd] = w.view(out_f, heads, hd)
    return p.view(out_f, heads * hd_pad)


class LuminaBlock(nn.Module):
    """JointTransformerBlock: attention + SwiGLU FFN with sandwich RMSNorms and tanh gates
    (modulation=True), or plain residuals (context refiner, modulation=False)."""

    def __init__(self, dim, heads, kv_heads, ffn_hidden, mode, device, gen=None, modulation=True, norm_eps=1e-5,
                 hd_pad=None):
        super().__init__()
        self.dim, self.heads, self.kv_heads = dim, heads, kv_heads
        self.hd = dim // heads
        self.hd_pad = hd_pad or self.hd   # attention head width (wider only to test zero padding)
        self.ffn = ffn_hidden
        self.modulation = modulation
        self.eps = norm_eps
        self.qkv = _rand_qlin(dim, (heads + 2 * kv_heads) * self.hd, mode, device, gen, bias=False)
        self.wo = _qlin(pad_head_columns(_rand_weight(dim, heads * self.hd, device, gen), heads, self.hd,
                                         self.hd_pad), None, mode)
        w1 = _rand_weight(ffn_hidden, dim, device, gen)
        w3 = _rand_weight(ffn_hidden, dim, device, gen)
        self.w13 = _qlin(glu_interleave(w1, w3), None, mode)
        del w1, w3
        self.w2 = _rand_qlin(ffn_hidden, dim, mode, device, gen, bias=False)
        one = lambda n: torch.ones(n, device=device, dtype=torch.bfloat16)  # noqa: E731
        self.q_norm, self.k_norm = one(self.hd), one(self.hd)
        self.attention_norm1, self.attention_norm2 = one(dim), one(dim)
        self.ffn_norm1, self.ffn_norm2 = one(dim), one(dim)

    def mod_slices(self, mod: torch.Tensor | None):
        """scale_msa, gate_msa, scale_mlp, gate_mlp (model.py:84-86) or all None."""
        if mod is None:
            return None, None, None, None
        D = self.dim
        return mod[:, 0:D], mod[:, D:2 * D], mod[:, 2 * D:3 * D], mod[:, 3 * D:4 * D]

    def forward(self, x: torch.Tensor, h: torch.Tensor, mod: torch.Tensor | None, freqs: torch.Tensor,
                next_norm: torch.Tensor | None, next_scale: torch.Tensor | None, next_eps: float):
        """x [B, L, dim] residual stream (updated in place); h [B*L, dim] = this block's
        attention_norm1(x) * (1 + scale_msa), overwritten with the next block's input
        (next_norm / next_scale / next_eps; next_norm None = last block)."""
        B, L, D = x.shape
        x2 = x.view(-1, D)
        H, Hk, hp = self.heads, self.kv_heads, self.hd_pad
        _, g_msa, s_mlp, g_mlp = self.mod_slices(mod)
        qkv = self.qkv.run(h, None)
        q = torch.empty(B, L, H, hp, dtype=torch.bfloat16, device=x.device)
        k = torch.empty(B, L, Hk, hp, dtype=torch.bfloat16, device=x.device)
        v = torch.empty(B, L, Hk, hp, dtype=torch.bfloat16, device=x.device)
        qkv_norm_rope(qkv.view(B, L, -1), H, self.q_norm, self.k_norm, freqs, q, k, v, eps=1e-6, Hkv=Hk)
        o = sageattn(q, k, v, tensor_layout="NHD", sm_scale=1.0 / math.sqrt(self.hd))
        y = self.wo.run(o.view(B * L, H * hp), None)
        rms_gate_residual(x2, y, h, L, self.attention_norm2, self.eps, g_msa, False, self.ffn_norm1, self.eps, s_mlp)
        f = self.w13.run(h, None, glu=True)
        y = self.w2.run(f, None)
        rms_gate_residual(x2, y, h if next_norm is not None else None, L, self.ffn_norm2, self.eps, g_mlp, False,
                          next_norm, next_eps, next_scale)
        return x


class LuminaDiT(nn.Module):
    """Lumina-Image-2.0 2B shape.  forward(img [B, L_img, p*p*C] patch tokens, t [B],
    cap [B, L_cap, cap_dim], ids [B, L_cap + L_img, 3]) -> [B, L_img, p*p*C]."""

    def __init__(self, dim=2304, n_layers=26, n_refiner=2, heads=24, kv_heads=8, ffn_hidden=6144, cap_dim=2304,
                 patch_dim=64, axes_dim=(32, 32, 32), norm_eps=1e-5, mode="int8", device="cuda", seed=0):
        super().__init__()
        gen = torch.Generator(device=device).manual_seed(seed)
        self.dim, self.axes_dim, self.eps = dim, axes_dim, norm_eps
        self.heads, self.kv_heads = heads, kv_heads
        tdim = min(dim, 1024)
        self.tdim = tdim
        blk = lambda m: LuminaBlock(dim, heads, kv_heads, ffn_hidden, mode, device, gen, m, norm_eps)  # noqa: E731
        self.x_embedder = _rand_qlin(patch_dim, dim, mode, device, gen)
        self.noise_refiner = nn.ModuleList([blk(True) for _ in range(n_refiner)])
        self.context_refiner = nn.ModuleList([blk(False) for _ in range(n_refiner)])
        self.t_mlp1 = _rand_qlin(256, tdim, mode, device, gen)
        self.t_mlp2 = _rand_qlin(tdim, tdim, mode, device, gen)
        self.cap_norm = torch.ones(cap_dim, device=device, dtype=torch.bfloat16)
        self.cap_linear = _rand_qlin(cap_dim, dim, mode, device, gen)
        self.layers = nn.ModuleList([blk(True) for _ in range(n_layers)])
        # every adaLN modulation linear reads the same silu(t): one stacked GEMM per step
        # (noise refiner blocks, main layers, then the final layer's scale)
        n_mod = n_refiner + n_layers
        ws = [_rand_weight(4 * dim, tdim, device, gen) for _ in range(n_mod)] + [_rand_weight(dim, tdim, device, gen)]
        bs = [((torch.rand(w.shape[0], device=device, generator=gen) * 2 - 1) / math.sqrt(tdim)).to(torch.bfloat16)
              for w in ws]
        self.adaLN = _qlin(torch.cat(ws), torch.cat(bs), mode)
        del ws
        self.final_linear = _rand_qlin(dim, patch_dim, mode, device, gen)

    @staticmethod
    def timestep_embedding(t: torch.Tensor, dim: int = 256, max_period: float = 10000.0) -> torch.Tensor:
        # LuminaTimestepEmbedder.timestep_embedding (model.py:15-28)
        half = dim // 2
        freqs = torch.exp(-math.log(max_period) * torch.arange(half, device=t.device, dtype=torch.float32) / half)
        args = t.float()[:, None] * freqs[None]
        return torch.cat([torch.cos(args), torch.sin(args)], dim=-1).to(torch.bfloat16)

    @staticmethod
    def position_ids(B: int, cap_len: int, h: int, w: int, device) -> torch.Tensor:
        """patchify_and_embed's ids (model.py:307-330): caption token i -> (i, 0, 0); image
        token (r, c) -> (cap_len, r, c)."""
        ids = torch.zeros(B, cap_len + h * w, 3, dtype=torch.int32, device=device)
        ids[:, :cap_len, 0] = torch.arange(cap_len, device=device, dtype=torch.int32)
        ids[:, cap_len:, 0] = cap_len
        ids[:, cap_len:, 1] = torch.arange(h, device=device, dtype=torch.int32).repeat_interleave(w)
        ids[:, cap_len:, 2] = torch.arange(w, device=device, dtype=torch.int32).repeat(h)
        return ids

    def _run(self, blocks, x, mods, freqs, tail_norm=None, tail_scale=None, tail_eps=None):
        """A chain of blocks on x [B, L, dim]; returns the input h of whatever follows the
        chain (tail_norm/tail_scale) or None."""
        B, L, D = x.shape
        x2 = x.view(-1, D)
        h = torch.empty_like(x2)
        b0 = blocks[0]
        s0 = b0.mod_slices(mods[0])[0]
        rms_gate_residual(x2, None, h, L, w_pre=b0.attention_norm1, eps_pre=b0.eps, scale=s0)
        for i, blk in enumerate(blocks):
            if i + 1 < len(blocks):
                nb = blocks[i + 1]
                nn_, ns, ne = nb.attention_norm1, nb.mod_slices(mods[i + 1])[0], nb.eps
            else:
                nn_, ns, ne = tail_norm, tail_scale, tail_eps
            blk(x, h, mods[i], freqs, nn_, ns, ne)
        return h if tail_norm is not None else None

    def forward(self, img: torch.Tensor, t: torch.Tensor, cap: torch.Tensor, freqs: torch.Tensor) -> torch.Tensor:
        B, Li, _ = img.shape
        Lc = cap.shape[1]
        D = self.dim
        temb = self.t_mlp2(F.silu(self.t_mlp1(self.timestep_embedding(t))))  # [B, tdim]
        mods_all = self.adaLN(F.silu(temb))  # [B, (n_mod * 4 + 1) * dim]
        # tanh of every gate once per step, in bf16 like the reference's gate.tanh()
        # (model.py:87, 94); the fused residual pass then takes the gates as they are
        n_mod_all = (mods_all.shape[1] - D) // (4 * D)
        mods_all[:, :4 * D * n_mod_all].view(B, n_mod_all, 4, D)[:, :, 1::2].tanh_()
        n_ref = len(self.noise_refiner)
        mod = lambda i: mods_all[:, 4 * D * i:4 * D * (i + 1)]  # noqa: E731
        # caption embedder: RMSNorm + linear (model.py:210-212)
        cap2 = cap.reshape(-1, cap.shape[-1]).contiguous()
        hc = torch.empty_like(cap2)
        rms_gate_residual(cap2, None, hc, Lc, w_pre=self.cap_norm, eps_pre=self.eps)
        xc = self.cap_linear.run(hc, None).view(B, Lc, D)
        xi = self.x_embedder(img.reshape(-1, img.shape[-1])).view(B, Li, D)
        # refiners on their own token ranges (model.py:336-366)
        self._run(self.context_refiner, xc, [None] * len(self.context_refiner), freqs[:, :Lc])
        self._run(self.noise_refiner, xi, [mod(i) for i in range(n_ref)], freqs[:, Lc:])
        x = torch.cat([xc, xi], dim=1)  # joint sequence [caption | image]
        n_main = len(self.layers)
        fscale = mods_all[:, 4 * D * (n_ref + n_main):4 * D * (n_ref + n_main) + D]
        self._run(self.layers, x, [mod(n_ref + i) for i in range(n_main)], freqs)
        # final layer: LayerNorm (no affine, eps 1e-6) * (1 + scale) -> linear (nextdit.py:63-78)
        fmod = torch.zeros(B, 2 * D, dtype=torch.bfloat16, device=x.device)  # [shift = 0 | scale]
        fmod[:, D:] = fscale
        hf = ln_modulate(x[:, Lc:].reshape(B * Li, D), fmod[:, :D], fmod[:, D:], Li)
        return self.final_linear.run(hf, None).view(B, Li, -1)

    def make_freqs(self, B: int, cap_len: int, h: int, w: int, device) -> torch.Tensor:
        return rope_freqs(self.position_ids(B, cap_len, h, w, device), self.axes_dim)


def lumina_step_flops(B: int = 1, L_img: int = 4096, L_cap: int = 256, dim: int = 2304, n_layers: int = 26,
                      n_refiner: int = 2, heads: int = 24, kv_heads: int = 8, ffn_hidden: int = 6144) -> float:
    """Algorithmic FLOPs of one Lumina-shaped forward (linears + attention at head_dim 96)."""
    hd = dim // heads
    per_tok = 2.0 * dim * ((heads + 2 * kv_heads) * hd + dim + 3 * ffn_hidden)
    attn = lambda L: 4.0 * L * L * hd * heads  # noqa: E731
    L = L_img + L_cap
    f = n_layers * (L * per_tok + attn(L))
    f += n_refiner * (L_img * per_tok + attn(L_img))
    f += n_refiner * (L_cap * per_tok + attn(L_cap))
    return B * f
