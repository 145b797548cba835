"""GPU: the Flux-shaped DiT forward built from the B200 ops against a float reference
of the same (dequantized) weights, and one Flux-dev-sized step at 4608 tokens."""
import math

import numpy as np
import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


def deq(ql):
    from oracle.numerics import e4m3_bits_to_f32

    codes = ql.codes.cpu().numpy()
    w = e4m3_bits_to_f32(codes.view(np.uint8)) if ql.mode != "int8" else codes.astype(np.float32)
    return torch.from_numpy(w).double().cuda() * ql.scale.double()[:, None]


def lin(ql, x):
    y = x.double() @ deq(ql).T
    return y + ql.bias.double() if ql.bias is not None else y


def ref_forward(m, img, txt, t, y, freqs):
    """Float64 restatement of FluxDiT.forward (torch ops only, SDPA attention)."""
    ln = lambda x: F.layer_norm(x, (x.shape[-1],), eps=1e-6)  # noqa: E731
    mod = lambda x, s, c: x * (1 + c) + s  # noqa: E731
    rms = lambda x: x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + 1e-6)  # noqa: E731

    def rope(x):
        xc = torch.view_as_complex(x.reshape(*x.shape[:-1], -1, 2).contiguous())
        return torch.view_as_real(xc * freqs.to(torch.complex128)[:, :, None]).flatten(-2)

    def attn(qkv, H, D):
        B, L, _ = qkv.shape
        q, k, v = qkv.view(B, L, 3, H, D).unbind(2)
        q, k = rope(rms(q)), rope(rms(k))
        o = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2))
        return o.transpose(1, 2)

    img, txt = lin(m.img_in, img), lin(m.txt_in, txt)
    vec = lin(m.time_in2, F.silu(lin(m.time_in1, m.timestep_embedding(t).double())))
    vec = vec + lin(m.vec_in2, F.silu(lin(m.vec_in1, y.double())))
    T = txt.shape[1]
    for b in m.double_blocks:
        im = lin(b.img_mod, F.silu(vec)).unsqueeze(1).chunk(6, -1)
        tm = lin(b.txt_mod, F.silu(vec)).unsqueeze(1).chunk(6, -1)
        iqkv = lin(b.img_qkv, mod(ln(img), im[0], im[1]))
        tqkv = lin(b.txt_qkv, mod(ln(txt), tm[0], tm[1]))
        a = attn(torch.cat([tqkv, iqkv], 1), b.heads, b.hd).reshape(img.shape[0], -1, b.dim)
        ta, ia = a[:, :T], a[:, T:]
        img = img + im[2] * lin(b.img_proj, ia)
        img = img + im[5] * lin(b.img_mlp2, F.gelu(lin(b.img_mlp1, mod(ln(img), im[3], im[4])), approximate="tanh"))
        txt = txt + tm[2] * lin(b.txt_proj, ta)
        txt = txt + tm[5] * lin(b.txt_mlp2, F.gelu(lin(b.txt_mlp1, mod(ln(txt), tm[3], tm[4])), approximate="tanh"))
    x = torch.cat([txt, img], 1)
    for b in m.single_blocks:
        s, c, g = lin(b.mod, F.silu(vec)).unsqueeze(1).chunk(3, -1)
        xm = mod(ln(x), s, c)
        qkv, mlp = lin(b.linear1_qkv, xm), lin(b.linear1_mlp, xm)
        a = attn(qkv, b.heads, b.hd).reshape(x.shape[0], -1, b.dim)
        x = x + g * lin(b.linear2, torch.cat([a, F.gelu(mlp, approximate="tanh")], -1))
    img = x[:, T:]
    s, c = lin(m.final_mod, F.silu(vec)).unsqueeze(1).chunk(2, -1)
    return lin(m.final, mod(ln(img), s, c))


@pytest.mark.parametrize("mode", ["fp8_w8a8", "int8"])
def test_small_flux_forward_vs_float_reference(cuda, mode):
    from quantfun2_b200.dit import FluxDiT, flux_position_ids, rope_freqs

    m = FluxDiT(dim=512, heads=4, depth_double=2, depth_single=2, mode=mode, device="cuda", seed=1,
                axes_dim=(16, 56, 56))
    g = torch.Generator(device="cuda").manual_seed(2)
    B, T, h, w = 2, 64, 12, 16
    img = torch.randn(B, h * w, 64, device="cuda", generator=g).bfloat16()
    txt = torch.randn(B, T, 4096, device="cuda", generator=g).bfloat16()
    t = torch.rand(B, device="cuda", generator=g)
    y = torch.randn(B, 768, device="cuda", generator=g).bfloat16()
    freqs = rope_freqs(flux_position_ids(B, T, h, w, "cuda"), (16, 56, 56))
    out = m(img, txt, t, y, freqs).float()
    ref = ref_forward(m, img, txt, t, y, freqs).float()
    cos = F.cosine_similarity(out.flatten(), ref.flatten(), dim=0).item()
    print(f"{mode}: cos={cos:.6f}")
    assert torch.isfinite(out).all() and cos > (0.995 if mode == "int8" else 0.98)


def test_flux_dev_size_step_runs(cuda):
    """One Flux-dev-sized step (19 + 38 blocks, hidden 3072, 4096 img + 512 txt tokens)."""
    from quantfun2_b200.dit import FluxDiT, flux_position_ids, rope_freqs

    m = FluxDiT(device="cuda", seed=0)
    g = torch.Generator(device="cuda").manual_seed(0)
    img = torch.randn(1, 4096, 64, device="cuda", generator=g).bfloat16()
    txt = torch.randn(1, 512, 4096, device="cuda", generator=g).bfloat16()
    freqs = rope_freqs(flux_position_ids(1, 512, 64, 64, "cuda"), (16, 56, 56))
    out = m(img, txt, torch.rand(1, device="cuda"), torch.randn(1, 768, device="cuda").bfloat16(), freqs)
    torch.cuda.synchronize()
    assert out.shape == (1, 4096, 64) and torch.isfinite(out.float()).all()
