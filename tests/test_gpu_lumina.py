"""GPU: the Lumina-shaped path — SwiGLU GEMM epilogue, the fused gated-residual /
RMSNorm-modulate pass, GQA + head-dim-padded q/k norm + RoPE, a small Lumina forward
against a float64 restatement of the same (dequantized) weights, and one 2B-sized step."""
import math

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


def _bf16_ulp(x: torch.Tensor) -> torch.Tensor:
    """Spacing of bf16 numbers at |x| (8 significant bits)."""
    e = torch.floor(torch.log2(x.abs().clamp_min(1e-30)))
    return torch.pow(2.0, e - 7)


def deq(ql):
    w = ql.codes.double()
    return w * ql.scale.double()[:, None]


def lin(ql, x):
    y = x.double() @ deq(ql).T
    return y + ql.bias.double() if ql.bias is not None else y


def test_gemm_swiglu_epilogue(cuda):
    from quantfun2_b200.quant import gemm, glu_interleave

    g = torch.Generator(device="cuda").manual_seed(0)
    M, K, Hd = 300, 320, 384
    a = torch.randn(M, K, device="cuda", generator=g).bfloat16()
    w1 = (torch.randn(Hd, K, device="cuda", generator=g) / 16).bfloat16()
    w3 = (torch.randn(Hd, K, device="cuda", generator=g) / 16).bfloat16()
    cs1 = torch.rand(Hd, device="cuda", generator=g) + 0.5
    cs3 = torch.rand(Hd, device="cuda", generator=g) + 0.5
    b1 = torch.randn(Hd, device="cuda", generator=g).bfloat16()
    b3 = torch.randn(Hd, device="cuda", generator=g).bfloat16()
    out = gemm(a, glu_interleave(w1, w3), col_scale=glu_interleave(cs1, cs3), bias=glu_interleave(b1, b3), glu=True)
    gt = (a.double() @ w1.double().T) * cs1.double() + b1.double()
    up = (a.double() @ w3.double().T) * cs3.double() + b3.double()
    ref = gt * torch.sigmoid(gt) * up
    err = (out.double() - ref).abs()
    # one bf16 rounding + SFU tanh (2^-11 absolute) + fp32 accumulation of K products
    bound = 2 * _bf16_ulp(ref) + 1e-3 * (gt.abs() + 1) * up.abs() + 1e-5 * (gt.abs() + 1) * (up.abs() + 1)
    assert out.shape == (M, Hd)
    bad = (err > bound).nonzero()
    if len(bad):
        i, j = bad[0].tolist()
        pytest.fail(f"{len(bad)} elements out of bound; first at ({i}, {j}): out {out[i, j].item()} ref "
                    f"{ref[i, j].item()} gate {gt[i, j].item()} up {up[i, j].item()} max err {err.max().item()}")


def test_rms_gate_residual(cuda):
    from quantfun2_b200.kernels import rms_gate_residual

    g = torch.Generator(device="cuda").manual_seed(1)
    B, L, D = 2, 37, 768
    x = torch.randn(B * L, D, device="cuda", generator=g).bfloat16()
    y = (torch.randn(B * L, D, device="cuda", generator=g) * 3).bfloat16()
    mod = torch.randn(B, 4 * D, device="cuda", generator=g).bfloat16()
    wpost = (torch.rand(D, device="cuda", generator=g) + 0.5).bfloat16()
    wpre = (torch.rand(D, device="cuda", generator=g) + 0.5).bfloat16()
    gate, scale = mod[:, D:2 * D], mod[:, 2 * D:3 * D]
    x0 = x.clone()
    h = torch.empty_like(x)
    rms_gate_residual(x, y, h, L, wpost, 1e-5, gate, True, wpre, 1e-5, scale)
    bidx = torch.arange(B * L, device="cuda") // L
    yd = y.double()
    yn = yd * torch.rsqrt(yd.pow(2).mean(-1, keepdim=True) + 1e-5) * wpost.double()
    xr = x0.double() + torch.tanh(gate.double())[bidx] * yn
    # one bf16 rounding of x + the SFU tanh (tanh.approx.f32, ~2^-11 relative)
    assert bool(((x.double() - xr).abs() <= _bf16_ulp(xr) * 1.01 + 6e-4 * yn.abs() + 1e-6).all())
    # with gates given as they are (gate_tanh=False) the only rounding is the bf16 store
    x1 = x0.clone()
    rms_gate_residual(x1, y, None, L, wpost, 1e-5, gate, False)
    xr1 = x0.double() + gate.double()[bidx] * yn
    assert bool(((x1.double() - xr1).abs() <= _bf16_ulp(xr1) * 1.01 + 1e-6).all())
    xd = x.double()  # h is defined on the stored (rounded) x
    hr = xd * torch.rsqrt(xd.pow(2).mean(-1, keepdim=True) + 1e-5) * wpre.double() * (1 + scale.double()[bidx])
    assert bool(((h.double() - hr).abs() <= _bf16_ulp(hr) * 1.01 + 1e-6).all())
    # norm-only form (caption embedder) leaves x alone
    h2 = torch.empty_like(x)
    xs = x.clone()
    rms_gate_residual(x, None, h2, L, w_pre=wpre, eps_pre=1e-5)
    assert torch.equal(x, xs)
    hr2 = xd * torch.rsqrt(xd.pow(2).mean(-1, keepdim=True) + 1e-5) * wpre.double()
    assert bool(((h2.double() - hr2).abs() <= _bf16_ulp(hr2) * 1.01 + 1e-6).all())


def test_qkv_norm_rope_gqa_padded(cuda):
    from quantfun2_b200.dit import rope_freqs
    from quantfun2_b200.kernels import qkv_norm_rope
    from quantfun2_b200.lumina import LuminaDiT

    g = torch.Generator(device="cuda").manual_seed(2)
    B, Lc, h, w, H, Hk, D = 2, 8, 6, 5, 6, 2, 96
    L = Lc + h * w
    qkv = torch.randn(B, L, (H + 2 * Hk) * D, device="cuda", generator=g).bfloat16()
    qw = (torch.rand(D, device="cuda", generator=g) + 0.5).bfloat16()
    kw = (torch.rand(D, device="cuda", generator=g) + 0.5).bfloat16()
    freqs = rope_freqs(LuminaDiT.position_ids(B, Lc, h, w, "cuda"), (32, 32, 32))
    q = torch.full((B, L, H, 128), 7.0, device="cuda").bfloat16()
    k = torch.full((B, L, Hk, 128), 7.0, device="cuda").bfloat16()
    v = torch.full((B, L, Hk, 128), 7.0, device="cuda").bfloat16()
    qkv_norm_rope(qkv, H, qw, kw, freqs, q, k, v, eps=1e-6, Hkv=Hk)
    x = qkv.double().view(B, L, H + 2 * Hk, D)
    f = freqs.to(torch.complex128)[:, :, None]

    def ref(t, wt):
        t = t * torch.rsqrt(t.pow(2).mean(-1, keepdim=True) + 1e-6) * wt.double()
        tc = torch.view_as_complex(t.reshape(*t.shape[:-1], -1, 2).contiguous())
        return torch.view_as_real(tc * f).flatten(-2)

    for got, exp in ((q, ref(x[:, :, :H], qw)), (k, ref(x[:, :, H:H + Hk], kw))):
        err = (got[..., :D].double() - exp).abs()
        assert bool((err <= 2 * _bf16_ulp(exp) + 1e-6).all()), err.max().item()
        assert bool((got[..., D:] == 0).all())
    assert torch.equal(v[..., :D], qkv.view(B, L, H + 2 * Hk, D)[:, :, H + Hk:])
    assert bool((v[..., D:] == 0).all())


def ref_lumina(m, img, t, cap, freqs):
    """Float64 restatement of LuminaDiT.forward (model.py:31-102, 392-414) on the
    dequantized weights, SDPA attention with GQA."""
    D, eps = m.dim, m.eps
    rms = lambda x, w, e: x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + e) * w.double()  # noqa: E731
    fr = freqs.to(torch.complex128)

    def rope(x, f):
        xc = torch.view_as_complex(x.reshape(*x.shape[:-1], -1, 2).contiguous())
        return torch.view_as_real(xc * f[:, :, None]).flatten(-2)

    def attention(b, hin, f):
        B, L, _ = hin.shape
        H, Hk, hd = b.heads, b.kv_heads, b.hd
        qkv = lin(b.qkv, hin)
        q = qkv[..., :H * hd].reshape(B, L, H, hd)
        k = qkv[..., H * hd:(H + Hk) * hd].reshape(B, L, Hk, hd)
        v = qkv[..., (H + Hk) * hd:].reshape(B, L, Hk, hd)
        q, k = rope(rms(q, b.q_norm, 1e-6), f), rope(rms(k, b.k_norm, 1e-6), f)
        rep = H // Hk
        k, v = k.repeat_interleave(rep, 2), v.repeat_interleave(rep, 2)
        o = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2),
                                           scale=1 / math.sqrt(hd)).transpose(1, 2)
        op = torch.zeros(B, L, H, b.hd_pad, dtype=torch.float64, device=o.device)
        op[..., :hd] = o
        return lin(b.wo, op.reshape(B, L, -1))

    def ffn(b, hin):
        y = lin(b.w13, hin)
        y = y.view(*y.shape[:-1], -1, 2, 128)
        gt, up = y[..., 0, :], y[..., 1, :]
        return lin(b.w2, (F.silu(gt) * up).flatten(-2))

    def block(b, x, mod, f):
        if mod is None:
            x = x + rms(attention(b, rms(x, b.attention_norm1, eps), f), b.attention_norm2, eps)
            return x + rms(ffn(b, rms(x, b.ffn_norm1, eps)), b.ffn_norm2, eps)
        s1, g1, s2, g2 = (c[:, None] for c in mod.chunk(4, -1))
        x = x + torch.tanh(g1) * rms(attention(b, rms(x, b.attention_norm1, eps) * (1 + s1), f), b.attention_norm2,
                                     eps)
        return x + torch.tanh(g2) * rms(ffn(b, rms(x, b.ffn_norm1, eps) * (1 + s2)), b.ffn_norm2, eps)

    temb = lin(m.t_mlp2, F.silu(lin(m.t_mlp1, m.timestep_embedding(t).double())))
    mods = lin(m.adaLN, F.silu(temb))
    Lc = cap.shape[1]
    xc = lin(m.cap_linear, rms(cap.double(), m.cap_norm, eps))
    xi = lin(m.x_embedder, img.double())
    for b in m.context_refiner:
        xc = block(b, xc, None, fr[:, :Lc])
    nr = len(m.noise_refiner)
    for i, b in enumerate(m.noise_refiner):
        xi = block(b, xi, mods[:, 4 * D * i:4 * D * (i + 1)], fr[:, Lc:])
    x = torch.cat([xc, xi], 1)
    for i, b in enumerate(m.layers):
        x = block(b, x, mods[:, 4 * D * (nr + i):4 * D * (nr + i + 1)], fr)
    n = nr + len(m.layers)
    fs = mods[:, 4 * D * n:4 * D * n + D][:, None]
    xf = F.layer_norm(x[:, Lc:], (D,), eps=1e-6) * (1 + fs)
    return lin(m.final_linear, xf)


def test_small_lumina_forward_vs_float_reference(cuda):
    from quantfun2_b200.lumina import LuminaDiT

    m = LuminaDiT(dim=768, n_layers=2, n_refiner=1, heads=8, kv_heads=4, ffn_hidden=512, cap_dim=768,
                  device="cuda", seed=3)
    g = torch.Generator(device="cuda").manual_seed(4)
    B, Lc, h, w = 2, 64, 16, 16
    img = torch.randn(B, h * w, 64, device="cuda", generator=g).bfloat16()
    cap = torch.randn(B, Lc, 768, device="cuda", generator=g).bfloat16()
    t = torch.rand(B, device="cuda", generator=g)
    freqs = m.make_freqs(B, Lc, h, w, "cuda")
    out = m(img, t, cap, freqs).float()
    ref = ref_lumina(m, img, t, cap, freqs).float()
    cos = F.cosine_similarity(out.flatten(), ref.flatten(), dim=0).item()
    print(f"lumina small: cos={cos:.6f} max_abs={(out - ref).abs().max().item():.4f}")
    assert out.shape == (B, h * w, 64)
    assert torch.isfinite(out).all() and cos > 0.995


def test_lumina_2b_size_step_runs(cuda):
    """One Lumina-Image-2.0-2B-sized step: 26 layers + 2 + 2 refiners, dim 2304, 24/8 heads
    of 96, SwiGLU 6144, 4096 image + 256 caption tokens."""
    from quantfun2_b200.lumina import LuminaDiT

    m = LuminaDiT(device="cuda", seed=0)
    g = torch.Generator(device="cuda").manual_seed(0)
    img = torch.randn(1, 4096, 64, device="cuda", generator=g).bfloat16()
    cap = torch.randn(1, 256, 2304, device="cuda", generator=g).bfloat16()
    out = m(img, torch.rand(1, device="cuda"), cap, m.make_freqs(1, 256, 64, 64, "cuda"))
    torch.cuda.synchronize()
    assert out.shape == (1, 4096, 64) and torch.isfinite(out.float()).all()
