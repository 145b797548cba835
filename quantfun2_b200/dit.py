"""Flux-dev- and Lumina-Image-2.0-shaped DiT forward passes built from the B200 ops.

These are the callers of the hot path (a7 / a10 in the reference): the block structure
follows src/models/flux/mmdit.py (DoubleStreamBlock :62-166, SingleStreamBlock
:169-231) and src/models/lumina/image_two/model.py (JointTransformerBlock :31-102,
JointAttention src/models/common/attn.py:133-236), with the defects of the reference's
Flux wiring corrected: txt tokens precede img tokens in the joint sequence, q/k reach
RoPE as [B, L, H, D] with complex frequencies, the attention output projection is the
block's own linear.  Weights are random (no checkpoints); every linear is a QLinear
(FP8 e4m3 W8A8 for Flux, INT8 weight-only for Lumina).  Attention runs the Sage
INT8/FP8 kernel.  The glue around it is fused into library kernels too: adaLN
LayerNorm + modulate (+ the e4m3 activation quantizer) in one row kernel, q/k RMSNorm +
RoPE in one kernel over the QKV projection, GELU / SwiGLU and the gated residual adds in
the GEMM epilogues, and Lumina's post-norm gated residual + pre-norm modulate in one
row kernel.

Sequence parallelism (Ulysses): with a process group of P ranks each rank holds L/P
tokens of the joint sequence; around attention an all-to-all turns [B, L/P, H, D]
into [B, L, H/P, D] and back (`ulysses_attention`).
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F
from torch import nn

from .attention import sageattn
from .kernels import copy_chunks, qkv_norm_rope, rmsnorm_apply, rope_apply_
from .quant import QLinear, quantize_rows


# ------------------------------------------------------------------ helpers --
def random_qlinear(in_f: int, out_f: int, mode: str, device, bias: bool = True, gen=None) -> QLinear:
    """A QLinear of random weights (uniform +-1/sqrt(in_f), the nn.Linear default)
    quantized on the device without materialising an fp32 copy."""
    bound = 1.0 / math.sqrt(in_f)
    w = (torch.rand(out_f, in_f, device=device, generator=gen) * 2 - 1).mul_(bound).to(torch.bfloat16)
    codes, scale = quantize_rows(w, "int8" if mode == "int8" else "e4m3")
    del w
    b = None
    if bias:
        b = ((torch.rand(out_f, device=device, generator=gen) * 2 - 1) * bound).to(torch.bfloat16)
    return QLinear(codes, scale, b, mode, in_f, out_f)


def layer_norm(x: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    return F.layer_norm(x, (x.shape[-1],), eps=eps)


def modulate(x: torch.Tensor, shift: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    # src/models/flux/mmdit.py:128 (modulate(x, scale) + shift)
    return torch.addcmul(shift, x, 1 + scale)


def rope_freqs(ids: torch.Tensor, axes_dim, theta: float = 10000.0) -> torch.Tensor:
    """Complex RoPE factors [B, L, sum(axes)/2] for integer positions ids [B, L, n_axes]
    (the per-axis construction of src/models/lumina/image_two/model.py:105-151)."""
    parts = []
    for i, d in enumerate(axes_dim):
        freqs = 1.0 / (theta ** (torch.arange(0, d, 2, dtype=torch.float64, device=ids.device) / d))
        ang = ids[..., i].to(torch.float64)[..., None] * freqs
        parts.append(torch.polar(torch.ones_like(ang), ang).to(torch.complex64))
    return torch.cat(parts, dim=-1)


def flux_position_ids(B: int, txt_len: int, h: int, w: int, device) -> torch.Tensor:
    """txt tokens at position 0 on every axis, then an (h, w) image grid (axis 0 = 0)."""
    ids = torch.zeros(B, txt_len + h * w, 3, dtype=torch.int32, device=device)
    r = torch.arange(h, device=device).repeat_interleave(w)
    c = torch.arange(w, device=device).repeat(h)
    ids[:, txt_len:, 1] = r
    ids[:, txt_len:, 2] = c
    return ids


# ------------------------------------------------------ sequence parallel --
class SeqParallel:
    """Ulysses all-to-all around attention.  group None = single GPU."""

    def __init__(self, group=None):
        self.group = group
        self.world = 1 if group is None else torch.distributed.get_world_size(group)

    def seq_to_heads(self, x: torch.Tensor) -> torch.Tensor:
        """[B, L/P, H, D] -> [B, L, H/P, D]"""
        if self.world == 1:
            return x
        B, Ls, H, D = x.shape
        P = self.world
        send = x.reshape(B, Ls, P, H // P, D).permute(2, 0, 1, 3, 4).contiguous()  # [P, B, Ls, H/P, D]
        recv = torch.empty_like(send)
        torch.distributed.all_to_all_single(recv, send, group=self.group)
        return recv.permute(1, 0, 2, 3, 4).reshape(B, P * Ls, H // P, D)

    def heads_to_seq(self, x: torch.Tensor) -> torch.Tensor:
        """[B, L, H/P, D] -> [B, L/P, H, D]"""
        if self.world == 1:
            return x
        B, L, Hp, D = x.shape
        P = self.world
        send = x.reshape(B, P, L // P, Hp, D).permute(1, 0, 2, 3, 4).contiguous()  # [P, B, L/P, H/P, D]
        recv = torch.empty_like(send)
        torch.distributed.all_to_all_single(recv, send, group=self.group)
        return recv.permute(1, 2, 0, 3, 4).reshape(B, L // P, P * Hp, D)


    def attention_packed(self, qkv3: torch.Tensor, out: torch.Tensor, attn_fn=None, permute=None) -> None:
        """qkv3 [B, L/P, 3, H, D] (q, k, v of this rank's tokens, contiguous) -> attention over
        the whole sequence written into out [B, L/P, H, D] (any strides, 16-byte rows).
        One all-to-all carries q, k and v together and one brings the output back; around
        them one copy packs the send buffer, one unpacks the received heads and one scatters
        the output heads.  attn_fn(q, k, v, o) writes o [B, L, H/P, D] (default: Sage);
        permute(dst, src, chunk_bytes, dims, src_strides, dst_strides) is the chunk copy
        (default: the qf2_copy_chunks kernel)."""
        attn_fn = attn_fn or (lambda a, b, c, o: sageattn(a, b, c, tensor_layout="NHD", out=o))
        B, Ls, _, H, D = qkv3.shape
        if self.world == 1:
            attn_fn(qkv3[:, :, 0], qkv3[:, :, 1], qkv3[:, :, 2], out)
            return
        P, Hp = self.world, H // self.world
        permute = permute or copy_chunks
        e = qkv3.element_size()
        hb = Hp * D * e                                   # bytes of one token's heads of one rank
        # [B, Ls, 3, P, Hp, D] -> [P, 3, B, Ls, Hp, D]: chunks of Hp*D, ordered (p, which, b, ls)
        send = torch.empty(P, 3, B, Ls, Hp, D, dtype=qkv3.dtype, device=qkv3.device)
        permute(send, qkv3, hb, (P, 3, B, Ls), (hb, P * hb, Ls * 3 * P * hb, 3 * P * hb),
                (3 * B * Ls * hb, B * Ls * hb, Ls * hb, hb))
        recv = torch.empty_like(send)
        torch.distributed.all_to_all_single(recv, send, group=self.group)
        # [P(src), 3, B, Ls, Hp, D] -> [3, B, P, Ls, Hp, D]: whole shards, token = src * Ls + local
        heads = torch.empty(3, B, P * Ls, Hp, D, dtype=qkv3.dtype, device=qkv3.device)
        sh = Ls * hb
        permute(heads, recv, sh, (3, B, P), (B * sh, sh, 3 * B * sh), (B * P * sh, P * sh, sh))
        # the output in the send order of the second exchange; for B = 1 [P, 1, Ls] is [1, L]
        o_send = torch.empty(P, B, Ls, Hp, D, dtype=out.dtype, device=out.device)
        if B == 1:
            attn_fn(heads[0], heads[1], heads[2], o_send.view(1, P * Ls, Hp, D))
        else:
            o = torch.empty(B, P * Ls, Hp, D, dtype=out.dtype, device=out.device)
            attn_fn(heads[0], heads[1], heads[2], o)
            permute(o_send, o, sh, (P, B), (sh, P * sh), (B * sh, sh))
        o_recv = torch.empty_like(o_send)
        torch.distributed.all_to_all_single(o_recv, o_send, group=self.group)
        # [P(src), B, Ls, Hp, D] -> out [B, Ls, P*Hp, D] (heads of rank p at [p*Hp, (p+1)*Hp))
        if out.stride(3) != 1:
            raise ValueError("out needs contiguous head_dim rows")
        ob, os_, oh = out.stride(0) * e, out.stride(1) * e, out.stride(2) * e
        if oh == D * e:  # a token's Hp heads are one contiguous chunk of out
            permute(out, o_recv, hb, (B, Ls, P), (Ls * hb, hb, B * Ls * hb), (ob, os_, hb))
        else:
            permute(out, o_recv, D * e, (B, Ls, P, Hp), (Ls * hb, hb, B * Ls * hb, D * e), (ob, os_, Hp * oh, oh))


def ulysses_attention(q, k, v, sp: SeqParallel, attn_fn=None) -> torch.Tensor:
    """q/k/v [B, L_local, H, D] (NHD) -> attention output [B, L_local, H, D]."""
    attn_fn = attn_fn or (lambda a, b, c: sageattn(a, b, c, tensor_layout="NHD"))
    qh, kh, vh = sp.seq_to_heads(q), sp.seq_to_heads(k), sp.seq_to_heads(v)
    return sp.heads_to_seq(attn_fn(qh, kh, vh))


def qk_norm_rope(qkv: torch.Tensor, H: int, D: int, qn: torch.Tensor, kn: torch.Tensor, freqs: torch.Tensor):
    """qkv [B, L, 3*H*D] -> q, k, v [B, L, H, D]: per-head RMSNorm (eps 1e-6) on q and k,
    then RoPE on q and k (rope_apply_ rotates in place)."""
    B, L, _ = qkv.shape
    q, k, v = qkv.view(B, L, 3, H, D).unbind(2)
    q = rmsnorm_apply(q, qn, 1e-6)
    k = rmsnorm_apply(k, kn, 1e-6)
    rope_apply_(q, k, freqs, fp16_trig=False)
    return q, k, v


# ---------------------------------------------------------------- Flux ------
class FluxDoubleBlock(nn.Module):
    """src/models/flux/mmdit.py:62-166 (img and txt streams, joint attention).
    adaLN LayerNorm+modulate is fused with the activation quantizer of the next linear;
    GELU and the gated residual adds run in the GEMM epilogues."""

    def __init__(self, dim, heads, mlp_ratio, mode, device, gen=None):
        super().__init__()
        self.dim, self.heads, self.hd = dim, heads, dim // heads
        mlp = int(dim * mlp_ratio)
        mk = lambda i, o: random_qlinear(i, o, mode, device, gen=gen)  # noqa: E731
        self.img_mod, self.txt_mod = mk(dim, 6 * dim), mk(dim, 6 * dim)
        self.img_qkv, self.txt_qkv = mk(dim, 3 * dim), mk(dim, 3 * dim)
        self.img_proj, self.txt_proj = mk(dim, dim), mk(dim, dim)
        self.img_mlp1, self.txt_mlp1 = mk(dim, mlp), mk(dim, mlp)
        self.img_mlp2, self.txt_mlp2 = mk(mlp, dim), mk(mlp, dim)
        ones = torch.ones(self.hd, device=device, dtype=torch.bfloat16)
        self.norms = [ones.clone() for _ in range(4)]  # img q, img k, txt q, txt k RMSNorm weights

    def _pre(self, x, mod, qkv_lin, qn, kn, freqs, q, k, v):
        """adaLN -> qkv projection -> fused q/k RMSNorm + RoPE into the joint q/k/v buffers."""
        B, L, D = x.shape
        a = qkv_lin.prep_ln_modulate(x.view(-1, D), mod[:, 0:D], mod[:, D:2 * D], L)
        qkv_norm_rope(qkv_lin.run(*a).view(B, L, -1), self.heads, qn, kn, freqs, q, k, v)

    def _post(self, x, attn_out, mod, proj, mlp1, mlp2):
        B, L, D = x.shape
        x2 = x.view(-1, D)
        # x += gate1 * proj(attn); x += gate2 * mlp2(gelu(mlp1(modulate(LN(x), shift2, scale2))))
        proj.run(*proj.prep(attn_out.reshape(-1, D)), out=x2, residual=x2, gate=mod[:, 2 * D:3 * D], rows_per_gate=L)
        h = mlp1.run(*mlp1.prep_ln_modulate(x2, mod[:, 3 * D:4 * D], mod[:, 4 * D:5 * D], L), gelu_col0=0)
        mlp2.run(*mlp2.prep(h), out=x2, residual=x2, gate=mod[:, 5 * D:6 * D], rows_per_gate=L)
        return x

    def forward(self, img, txt, vec, freqs, sp: SeqParallel, txt_local: int):
        B = img.shape[0]
        sv = F.silu(vec)
        im, tm = self.img_mod(sv), self.txt_mod(sv)  # [B, 6 * dim]
        T = txt_local
        L = T + img.shape[1]
        qkv3 = torch.empty(B, L, 3, self.heads, self.hd, dtype=torch.bfloat16, device=img.device)
        q, k, v = qkv3.unbind(2)
        self._pre(txt, tm, self.txt_qkv, self.norms[2], self.norms[3], freqs[:, :T], q[:, :T], k[:, :T], v[:, :T])
        self._pre(img, im, self.img_qkv, self.norms[0], self.norms[1], freqs[:, T:], q[:, T:], k[:, T:], v[:, T:])
        a = torch.empty(B, L, self.heads, self.hd, dtype=torch.bfloat16, device=img.device)
        sp.attention_packed(qkv3, a)
        a = a.view(B, L, self.dim)
        img = self._post(img, a[:, txt_local:], im, self.img_proj, self.img_mlp1, self.img_mlp2)
        txt = self._post(txt, a[:, :txt_local], tm, self.txt_proj, self.txt_mlp1, self.txt_mlp2)
        return img, txt


class FluxSingleBlock(nn.Module):
    """src/models/flux/mmdit.py:169-231 (fused qkv + MLP input, fused output).  linear_1 is
    held as its qkv and MLP row blocks; the MLP block writes GELU(.) and the attention writes
    its output straight into the two column ranges of linear_2's input, so no concat runs."""

    def __init__(self, dim, heads, mlp_ratio, mode, device, gen=None):
        super().__init__()
        self.dim, self.heads, self.hd = dim, heads, dim // heads
        self.mlp = int(dim * mlp_ratio)
        self.mod = random_qlinear(dim, 3 * dim, mode, device, gen=gen)
        self.linear1_qkv = random_qlinear(dim, 3 * dim, mode, device, gen=gen)
        self.linear1_mlp = random_qlinear(dim, self.mlp, mode, device, gen=gen)
        self.linear2 = random_qlinear(dim + self.mlp, dim, mode, device, gen=gen)
        self.qn = torch.ones(self.hd, device=device, dtype=torch.bfloat16)
        self.kn = torch.ones(self.hd, device=device, dtype=torch.bfloat16)

    def forward(self, x, vec, freqs, sp: SeqParallel):
        B, L, D = x.shape
        x2 = x.view(-1, D)
        mod = self.mod(F.silu(vec))  # [B, 3 * dim]: shift, scale, gate
        a = self.linear1_qkv.prep_ln_modulate(x2, mod[:, 0:D], mod[:, D:2 * D], L)
        qkv = self.linear1_qkv.run(*a)
        cat = torch.empty(B * L, D + self.mlp, dtype=torch.bfloat16, device=x.device)
        self.linear1_mlp.run(*a, out=cat[:, D:], gelu_col0=0)
        qkv3 = torch.empty(B, L, 3, self.heads, self.hd, dtype=torch.bfloat16, device=x.device)
        q, k, v = qkv3.unbind(2)
        qkv_norm_rope(qkv.view(B, L, -1), self.heads, self.qn, self.kn, freqs, q, k, v)
        sp.attention_packed(qkv3, cat[:, :D].view(B, L, self.heads, self.hd))
        self.linear2.run(*self.linear2.prep(cat), out=x2, residual=x2, gate=mod[:, 2 * D:3 * D], rows_per_gate=L)
        return x


class FluxDiT(nn.Module):
    """Flux-dev shape: 19 double + 38 single blocks, hidden 3072, 24 heads x 128, MLP x4,
    RoPE axes (16, 56, 56).  Inputs are token embeddings: img [B, L_img, 64] (2x2 patches of
    16 latent channels), txt [B, L_txt, 4096], timestep t [B], pooled text y [B, 768]."""

    def __init__(self, dim=3072, heads=24, depth_double=19, depth_single=38, mlp_ratio=4.0, mode="fp8_w8a8",
                 device="cuda", seed=0, axes_dim=(16, 56, 56)):
        super().__init__()
        gen = torch.Generator(device=device).manual_seed(seed)
        self.dim, self.heads, self.axes_dim = dim, heads, axes_dim
        mk = lambda i, o: random_qlinear(i, o, mode, device, gen=gen)  # noqa: E731
        self.img_in, self.txt_in = mk(64, dim), mk(4096, dim)
        self.time_in1, self.time_in2 = mk(256, dim), mk(dim, dim)
        self.vec_in1, self.vec_in2 = mk(768, dim), mk(dim, dim)
        self.double_blocks = nn.ModuleList([FluxDoubleBlock(dim, heads, mlp_ratio, mode, device, gen)
                                     for _ in range(depth_double)])
        self.single_blocks = nn.ModuleList([FluxSingleBlock(dim, heads, mlp_ratio, mode, device, gen)
                                     for _ in range(depth_single)])
        self.final_mod = mk(dim, 2 * dim)
        self.final = mk(dim, 64)

    @staticmethod
    def timestep_embedding(t: torch.Tensor, dim: int = 256, max_period: float = 10000.0) -> torch.Tensor:
        half = dim // 2
        freqs = torch.exp(-math.log(max_period) * torch.arange(half, device=t.device, dtype=torch.float32) / half)
        args = (1000.0 * t.float())[:, None] * freqs[None]
        return torch.cat([torch.cos(args), torch.sin(args)], dim=-1).to(torch.bfloat16)

    def forward(self, img, txt, t, y, freqs, sp: SeqParallel | None = None):
        """img/txt: this rank's shard of the image and text tokens (txt first in the joint
        sequence); freqs: complex RoPE factors of the rank's joint-sequence shard."""
        sp = sp or SeqParallel()
        img, txt = self.img_in(img).contiguous(), self.txt_in(txt).contiguous()
        vec = self.time_in2(F.silu(self.time_in1(self.timestep_embedding(t))))
        vec = vec + self.vec_in2(F.silu(self.vec_in1(y)))
        txt_local = txt.shape[1]
        for blk in self.double_blocks:
            img, txt = blk(img, txt, vec, freqs, sp, txt_local)
        x = torch.cat([txt, img], dim=1).contiguous()
        for blk in self.single_blocks:
            x = blk(x, vec, freqs, sp)
        img = x[:, txt_local:]
        shift, scale = self.final_mod(F.silu(vec)).unsqueeze(1).chunk(2, dim=-1)
        return self.final(modulate(layer_norm(img), shift, scale))


def flux_step_flops(L: int, dim: int = 3072, heads: int = 24, n_double: int = 19, n_single: int = 38,
                    mlp_ratio: float = 4.0) -> float:
    """Algorithmic FLOPs of one Flux-shaped forward at L joint tokens (linears + attention)."""
    mlp = int(dim * mlp_ratio)
    per_stream = dim * (3 * dim + dim + 2 * mlp)
    single = dim * (3 * dim + mlp) + (dim + mlp) * dim
    lin = 2.0 * L * (n_double * per_stream + n_single * single)
    attn = 4.0 * L * L * dim * (n_double + n_single)
    return lin + attn
