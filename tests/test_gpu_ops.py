"""GPU parity of RoPE / RMSNorm / softmax (libqf2b200.so) against the reference's golden
vectors and the oracle restatements."""
import numpy as np
import pytest
import torch

from oracle import ops
from oracle.numerics import bf16_bits_to_f32, f32_to_bf16_bits

pytestmark = pytest.mark.gpu


def t_bf16(bits, dev):
    return torch.from_numpy(bits.view(np.int16).copy()).view(torch.bfloat16).to(dev)


def bits(t):
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def cplx(a):
    return torch.view_as_complex(torch.from_numpy(np.ascontiguousarray(a)))


def test_rope_golden_f32(cuda, golden):
    from quantfun2_b200.kernels import rope_apply

    xq = torch.from_numpy(golden["rope_f32_xq"]).to(cuda)
    xk = torch.from_numpy(golden["rope_f32_xk"]).to(cuda)
    f = cplx(golden["rope_freqs"]).to(cuda)
    oq, ok = rope_apply(xq, xk, f)
    np.testing.assert_allclose(oq.cpu().numpy(), golden["rope_f32_oq"], rtol=0, atol=2e-6)
    np.testing.assert_allclose(ok.cpu().numpy(), golden["rope_f32_ok"], rtol=0, atol=2e-6)
    # bit-exact against the oracle restatement (same rounding steps)
    rq, rk = ops.rope_apply(golden["rope_f32_xq"], golden["rope_f32_xk"], cplx(golden["rope_freqs"]).numpy(), "f32")
    assert np.array_equal(oq.cpu().numpy(), rq) and np.array_equal(ok.cpu().numpy(), rk)


def test_rope_golden_bf16_and_inplace(cuda, golden):
    from quantfun2_b200.kernels import rope_apply, rope_apply_

    xq = t_bf16(golden["rope_bf16_xq"], cuda)
    xk = t_bf16(golden["rope_bf16_xk"], cuda)
    f = cplx(golden["rope_freqs"]).to(cuda)
    oq, ok = rope_apply(xq, xk, f)
    for got, ref in ((oq, golden["rope_bf16_oq"]), (ok, golden["rope_bf16_ok"])):
        d = np.abs(bits(got).astype(np.int32) - ref.astype(np.int32))
        assert d.max() <= 1 and (d == 0).mean() > 0.999
    # the Triton-path semantics: in place, fp16-rounded cos/sin
    q2, k2 = xq.clone(), xk.clone()
    r = rope_apply_(q2, k2, f)
    assert r[0].data_ptr() == q2.data_ptr()
    rq, rk = ops.rope_apply(bf16_bits_to_f32(golden["rope_bf16_xq"]), bf16_bits_to_f32(golden["rope_bf16_xk"]),
                            cplx(golden["rope_freqs"]).numpy(), "bf16", fp16_trig=True)
    assert np.array_equal(bits(q2), f32_to_bf16_bits(rq)) and np.array_equal(bits(k2), f32_to_bf16_bits(rk))


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_rope_strided_hnd_views_and_broadcast(cuda, dtype):
    """Flux passes q/k as [B, H, L, D] permuted views; freqs broadcast over batch."""
    from quantfun2_b200.kernels import rope_apply

    g = torch.Generator().manual_seed(3)
    B, H, L, D = 2, 3, 77, 128
    qh = torch.randn(B, H, L, D, generator=g).to(dtype)
    kh = torch.randn(B, H, L, D, generator=g).to(dtype)
    ang = torch.rand(1, L, D // 2, generator=g) * 6.28
    f = torch.polar(torch.ones_like(ang), ang)
    oq, ok = rope_apply(qh.to(cuda).permute(0, 2, 1, 3), kh.to(cuda).permute(0, 2, 1, 3), f.to(cuda))
    tag = {torch.bfloat16: "bf16", torch.float16: "f16", torch.float32: "f32"}[dtype]
    rq, rk = ops.rope_apply(qh.float().permute(0, 2, 1, 3).numpy(), kh.float().permute(0, 2, 1, 3).numpy(),
                            np.broadcast_to(f.numpy(), (B, L, D // 2)), tag)
    assert np.array_equal(oq.float().cpu().numpy(), rq)
    assert np.array_equal(ok.float().cpu().numpy(), rk)


@pytest.mark.parametrize("tag", ["head", "row"])
def test_rmsnorm_golden(cuda, golden, tag):
    from quantfun2_b200.kernels import rmsnorm_apply

    eps = float(golden[f"rms_{tag}_eps"][0])
    y = rmsnorm_apply(torch.from_numpy(golden[f"rms_{tag}_x_f32"]).to(cuda),
                      torch.from_numpy(golden[f"rms_{tag}_w_f32"]).to(cuda), eps)
    np.testing.assert_allclose(y.cpu().numpy(), golden[f"rms_{tag}_y_f32"], rtol=3e-6, atol=3e-6)
    yb = rmsnorm_apply(t_bf16(golden[f"rms_{tag}_x_bf16"], cuda), t_bf16(golden[f"rms_{tag}_w_bf16"], cuda), eps)
    assert yb.dtype == torch.bfloat16
    d = np.abs(bits(yb).astype(np.int32) - golden[f"rms_{tag}_y_bf16"].astype(np.int32))
    assert d.max() <= 1 and (d == 0).mean() > 0.99


@pytest.mark.parametrize("N", [64, 96, 128, 2304, 3072, 5000, 97])
@pytest.mark.parametrize("fused", [False, True])
def test_rmsnorm_shapes_vs_oracle(cuda, N, fused):
    from quantfun2_b200.kernels import rmsnorm_apply

    g = torch.Generator().manual_seed(N)
    x = (torch.randn(33, N, generator=g) * 2).bfloat16()
    w = (torch.rand(N, generator=g) + 0.5).bfloat16()
    y = rmsnorm_apply(x.to(cuda), w.to(cuda), 1e-6, fused=fused)
    r = ops.rmsnorm_apply(x.float().numpy(), w.float().numpy(), 1e-6, "bf16", fused=fused)
    d = np.abs(bits(y).astype(np.int32) - f32_to_bf16_bits(r).astype(np.int32))
    assert d.max() <= 1 and (d == 0).mean() > 0.99


def test_rmsnorm_mixed_dtypes(cuda):
    """bf16 activations with an fp32 weight promote to fp32 output, as the eager body does."""
    from quantfun2_b200.kernels import rmsnorm_apply

    g = torch.Generator().manual_seed(5)
    x = torch.randn(10, 96, generator=g).bfloat16()
    w = torch.rand(96, generator=g) + 0.5
    y = rmsnorm_apply(x.to(cuda), w.to(cuda), 1e-6)
    assert y.dtype == torch.float32
    r = ops.rmsnorm_apply(x.float().numpy(), w.numpy(), 1e-6, "bf16", out_dtype="f32")
    np.testing.assert_allclose(y.cpu().numpy(), r, rtol=1e-6, atol=1e-6)


def test_softmax_golden_and_long_rows(cuda, golden):
    from quantfun2_b200.kernels import inplace_softmax

    x = torch.from_numpy(golden["softmax_x_f32"]).to(cuda)
    y = inplace_softmax(x, -1)
    assert y.data_ptr() == x.data_ptr()
    np.testing.assert_allclose(y.cpu().numpy(), golden["softmax_y_f32"], rtol=1e-5, atol=1e-7)
    xb = t_bf16(golden["softmax_x_bf16"], cuda)
    yb = inplace_softmax(xb, -1)
    d = np.abs(bits(yb).astype(np.int32) - golden["softmax_y_bf16"].astype(np.int32))
    assert d.max() <= 1
    g = torch.Generator().manual_seed(9)
    z = torch.randn(3, 16400, generator=g) * 5
    z[1, 100:] = -float("inf")
    r = ops.softmax_lastdim(z.numpy())
    out = inplace_softmax(z.to(cuda)).cpu().numpy()
    np.testing.assert_allclose(out, r, rtol=1e-5, atol=1e-9)


@pytest.mark.parametrize("n,dtype", [(16384, torch.bfloat16), (2048, torch.float16), (8192, torch.float32),
                                     (96, torch.bfloat16), (4100, torch.float32)])
def test_softmax_register_rows(cuda, n, dtype):
    """Rows that fit one CTA's registers (read once, written once), with -inf entries and
    a -inf tail; within one ulp of the output dtype of the fp64 softmax (96 bf16 elements
    leave most threads of the CTA idle)."""
    from quantfun2_b200.kernels import inplace_softmax

    g = torch.Generator().manual_seed(n)
    z = (torch.randn(37, n, generator=g) * 4).to(dtype)
    z[3, n // 3:] = -float("inf")
    z[5, ::7] = -float("inf")
    ref = torch.softmax(z.double(), -1)
    out = inplace_softmax(z.to(cuda)).cpu()
    # one ulp of the output dtype relative to the value (fp32: the SFU exponential's error)
    ulp = {torch.bfloat16: 2.0 ** -7, torch.float16: 2.0 ** -10, torch.float32: 1e-5}[dtype]
    tiny = {torch.bfloat16: 1e-38, torch.float16: 2.0 ** -24, torch.float32: 1e-38}[dtype]  # underflow floor
    err = (out.double() - ref).abs()
    assert bool((err <= ulp * ref.abs() + tiny).all()), (err / ref.abs().clamp_min(1e-30)).max().item()


def test_qkv_norm_rope_fused(cuda):
    """Fused q/k RMSNorm + RoPE + v copy into offset views of joint buffers."""
    from quantfun2_b200.kernels import qkv_norm_rope

    g = torch.Generator().manual_seed(8)
    B, L, H, D, off = 2, 70, 3, 128, 5
    qkv = (torch.randn(B, L, 3 * H * D, generator=g) * 2).bfloat16()
    qw = (torch.rand(D, generator=g) + 0.5).bfloat16()
    kw = (torch.rand(D, generator=g) + 0.5).bfloat16()
    ang = torch.rand(B, L, D // 2, generator=g) * 6
    f = torch.polar(torch.ones_like(ang), ang)
    q, k, v = (torch.zeros(B, L + off, H, D, dtype=torch.bfloat16, device=cuda) for _ in range(3))
    qkv_norm_rope(qkv.to(cuda), H, qw.to(cuda), kw.to(cuda), f.to(cuda), q[:, off:], k[:, off:], v[:, off:])
    x = qkv.float().view(B, L, 3, H, D)

    def ref(t, w):
        n = t.double() * torch.rsqrt(t.double().pow(2).mean(-1, keepdim=True) + 1e-6) * w.double()
        c = torch.view_as_complex(n.reshape(B, L, H, D // 2, 2).contiguous()) * f.to(torch.complex128)[:, :, None]
        return torch.view_as_real(c).reshape(B, L, H, D)

    for got, want in ((q, ref(x[:, :, 0], qw)), (k, ref(x[:, :, 1], kw))):
        err = (got[:, off:].float().cpu().double() - want).abs().max().item()
        assert err < 0.02 * want.abs().max().item()
        assert not got[:, :off].any()
    assert torch.equal(v[:, off:].cpu(), qkv.view(B, L, 3, H, D)[:, :, 2])


@pytest.mark.parametrize("Ls", [40, 37])
def test_copy_chunks_ulysses_layouts(cuda, Ls):
    """qf2_copy_chunks against torch permute copies for the three layout changes around
    the head-parallel all-to-all (pack q/k/v per destination rank, unpack received
    shards, scatter output heads into a row-strided buffer); 768-byte chunks take the
    warp-per-chunk path, whole shards the segment path."""
    from quantfun2_b200.kernels import copy_chunks

    B, P, Hp, D = 2, 4, 3, 128
    e = 2
    hb = Hp * D * e
    qkv3 = torch.randn(B, Ls, 3, P * Hp, D, device=cuda).bfloat16()
    send = torch.empty(P, 3, B, Ls, Hp, D, device=cuda, dtype=torch.bfloat16)
    copy_chunks(send, qkv3, hb, (P, 3, B, Ls), (hb, P * hb, Ls * 3 * P * hb, 3 * P * hb),
                (3 * B * Ls * hb, B * Ls * hb, Ls * hb, hb))
    assert torch.equal(send, qkv3.view(B, Ls, 3, P, Hp, D).permute(3, 2, 0, 1, 4, 5))
    sh = Ls * hb
    heads = torch.empty(3, B, P * Ls, Hp, D, device=cuda, dtype=torch.bfloat16)
    copy_chunks(heads, send, sh, (3, B, P), (B * sh, sh, 3 * B * sh), (B * P * sh, P * sh, sh))
    assert torch.equal(heads, send.permute(1, 2, 0, 3, 4, 5).reshape(3, B, P * Ls, Hp, D))
    o_recv = torch.randn(P, B, Ls, Hp, D, device=cuda).bfloat16()
    big = torch.zeros(B, Ls, P * Hp * D + 64, device=cuda, dtype=torch.bfloat16)
    out = big[:, :, :P * Hp * D].view(B, Ls, P * Hp, D)
    copy_chunks(out, o_recv, hb, (B, Ls, P), (Ls * hb, hb, B * Ls * hb),
                (out.stride(0) * e, out.stride(1) * e, hb))
    assert torch.equal(out, o_recv.permute(1, 2, 0, 3, 4).reshape(B, Ls, P * Hp, D))
    assert not big[:, :, P * Hp * D:].any()  # nothing written past the rows
