"""GPU parity of the quantized linears: per-row quantizers bit-exact against the oracle;
tcgen05 GEMM and QLinear outputs within tolerance of fp64 references."""
import math

import numpy as np
import pytest
import torch

from oracle import qlinear as oq
from oracle.numerics import e4m3_bits_to_f32

pytestmark = pytest.mark.gpu


def rel_err(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-12))


@pytest.mark.parametrize("fmt", ["int8", "e4m3"])
def test_quantize_rows_bit_exact(cuda, fmt):
    from quantfun2_b200.quant import quantize_rows

    g = torch.Generator().manual_seed(0)
    w = (torch.randn(300, 520, generator=g) * torch.rand(300, 1, generator=g) * 3).bfloat16()
    w[7] = 0
    q, s = quantize_rows(w.to(cuda), fmt)
    ref_q, ref_s = (oq.quantize_rows_int8 if fmt == "int8" else oq.quantize_rows_e4m3)(w.float().numpy())
    assert np.array_equal(s.cpu().numpy(), ref_s)
    assert np.array_equal(q.cpu().numpy().view(np.uint8), ref_q.view(np.uint8))


@pytest.mark.parametrize("fmt", ["int8", "e4m3"])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16, torch.float32])
def test_quantize_weight_torchao_rule_bit_exact(cuda, fmt, dtype):
    """Weight quantizer of the reference's quantize-on-load (torchao 0.7.0 steps in the
    weight's dtype) against the restatement: codes and scales bit for bit, including an
    all-zero row and, in fp16, a row whose reciprocal scale overflows to inf."""
    from quantfun2_b200.quant import quantize_weight

    g = torch.Generator().manual_seed(1)
    w = (torch.randn(333, 1000, generator=g) * torch.rand(333, 1, generator=g) * 0.2).to(dtype)
    w[5] = 0
    w[9] = w[9] * 1e-3          # amax ~1e-4: fp16 scale ~1e-6 -> 1/scale overflows fp16
    q, s = quantize_weight(w.to(cuda), fmt)
    tag = {torch.float16: "f16", torch.bfloat16: "bf16", torch.float32: "f32"}[dtype]
    ref_q, ref_s = oq.quantize_weight_torchao(w.float().numpy(), fmt, tag)
    assert np.array_equal(s.cpu().numpy(), ref_s)
    assert np.array_equal(q.cpu().numpy().view(np.uint8), ref_q.view(np.uint8))


@pytest.mark.parametrize("mnk", [(128, 256, 64), (300, 776, 200), (2304, 3072, 1024)])
def test_gemm_fp16(cuda, mnk):
    """fp16 x fp16 operands (kind::f16 with the f16 format), fp16 and fp32 output."""
    from quantfun2_b200.quant import gemm

    M, N, K = mnk
    g = torch.Generator(device=cuda).manual_seed(M + 1)
    a = torch.randn(M, K, device=cuda, generator=g).half()
    b = torch.randn(N, K, device=cuda, generator=g).half()
    cs = torch.rand(N, device=cuda, generator=g) + 0.5
    bias = torch.randn(N, device=cuda, generator=g)
    ref = (a.double() @ b.double().T) * cs.double()[None, :] + bias.double()[None, :]
    d32 = gemm(a, b, col_scale=cs, bias=bias, out_dtype=torch.float32)
    assert rel_err(d32.cpu(), ref.cpu()) < 1e-5
    d16 = gemm(a, b, col_scale=cs, bias=bias, out_dtype=torch.float16)
    assert d16.dtype == torch.float16
    assert rel_err(d16.float().cpu(), ref.cpu()) < 1e-3


@pytest.mark.parametrize("mnk", [(128, 256, 64), (300, 776, 200), (4608, 3072, 3072), (257, 2304, 6144)])
def test_gemm_bf16(cuda, mnk):
    from quantfun2_b200.quant import gemm

    M, N, K = mnk
    g = torch.Generator(device=cuda).manual_seed(M)
    a = torch.randn(M, K, device=cuda, generator=g).bfloat16()
    b = torch.randn(N, K, device=cuda, generator=g).bfloat16()
    cs = torch.rand(N, device=cuda, generator=g) + 0.5
    bias = torch.randn(N, device=cuda, generator=g).bfloat16()
    d = gemm(a, b, col_scale=cs, bias=bias, out_dtype=torch.float32)
    ref = (a.double() @ b.double().T) * cs.double()[None, :] + bias.double()[None, :]
    assert rel_err(d.cpu(), ref.cpu()) < 1e-5
    d16 = gemm(a, b)
    assert rel_err(d16.float().cpu(), (a.double() @ b.double().T).cpu()) < 8e-3


@pytest.mark.parametrize("n", [2304, 3840, 1000, 384, 96])
@pytest.mark.parametrize("fp8", [False, True])
def test_gemm_pair_tile_widths(cuda, n, fp8):
    """CTA-pair path (M > 128) over output widths that select 256 / 192 / 128-column
    tiles and ragged last tiles; bf16 output through the TMA-store epilogue."""
    from quantfun2_b200.quant import gemm, quantize_rows

    M, K = 4352 + 40, 384
    g = torch.Generator(device=cuda).manual_seed(n)
    x = torch.randn(M, K, device=cuda, generator=g).bfloat16()
    w = torch.randn(n, K, device=cuda, generator=g).bfloat16()
    bias = torch.randn(n, device=cuda, generator=g).bfloat16()
    if fp8:
        xq, xs = quantize_rows(x, "e4m3")
        wq, ws = quantize_rows(w, "e4m3")
        d = gemm(xq, wq, row_scale=xs, col_scale=ws, bias=bias, fp8=True)
        xf = torch.from_numpy(e4m3_bits_to_f32(xq.cpu().numpy())).double().to(cuda) * xs.double()[:, None]
        wf = torch.from_numpy(e4m3_bits_to_f32(wq.cpu().numpy())).double().to(cuda) * ws.double()[:, None]
        ref = xf @ wf.T + bias.double()
    else:
        d = gemm(x, w, bias=bias)
        ref = x.double() @ w.double().T + bias.double()
    assert d.shape == (M, n)
    assert rel_err(d.float().cpu(), ref.cpu()) < 8e-3


def _random_codes(fmt, n, k, device, seed):
    g = torch.Generator().manual_seed(seed)
    if fmt == "int8":
        q = torch.randint(-128, 128, (n, k), generator=g, dtype=torch.int8)
        q[0, :4] = torch.tensor([-128, 127, 0, -1], dtype=torch.int8)
    else:
        q = torch.randint(0, 256, (n, k), generator=g, dtype=torch.int32).to(torch.uint8)
        q[(q & 0x7F) == 0x7F] = 0   # no NaN codes
        q[0, :6] = torch.tensor([0x7E, 0xFE, 0x01, 0x81, 0x08, 0x80], dtype=torch.uint8)  # +-448, subnormals, -0
    return q.to(device)


@pytest.mark.parametrize("fmt", ["int8", "e4m3"])
@pytest.mark.parametrize("act", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("mnk", [(1, 9216, 1024), (100, 776, 272), (300, 2304, 2304), (4392, 1000, 384),
                                 (4352, 2304, 2304)])
def test_gemm_codes_bit_exact_vs_converted(cuda, fmt, act, mnk):
    """Weight-code GEMM (codes converted to 16-bit in shared memory) against the 16-bit
    GEMM on the same codes converted beforehand: bit for bit, on the single-CTA (M <= 128)
    and CTA-pair kernels, ragged N and K tails, every code class (int8 extremes, e4m3
    +-448, subnormals, -0)."""
    from quantfun2_b200.quant import codes_to, gemm

    M, N, K = mnk
    g = torch.Generator(device=cuda).manual_seed(M + N)
    x = torch.randn(M, K, device=cuda, generator=g).to(act)
    q = _random_codes(fmt, N, K, cuda, N)
    sc = torch.rand(N, device=cuda, generator=g) * 0.01
    bias = torch.randn(N, device=cuda, generator=g).bfloat16()
    d = gemm(x, q, col_scale=sc, bias=bias, out_dtype=act, codes=fmt)
    ref = gemm(x, codes_to(q, fmt, act), col_scale=sc, bias=bias, out_dtype=act)
    assert torch.equal(d.view(torch.int16), ref.view(torch.int16))
    wf = codes_to(q, fmt, act).float()
    exact = (x.double() @ wf.double().T) * sc.double() + bias.double()
    assert rel_err(d.float().cpu(), exact.cpu()) < 1e-2


@pytest.mark.parametrize("fmt", ["int8", "e4m3"])
def test_gemm_codes_fused_epilogues(cuda, fmt):
    """The DiT epilogues on the weight-code kernel: SwiGLU (interleaved w1 / w3 codes) and
    GELU + gated residual in place, bit for bit against the converted-weight GEMM."""
    from quantfun2_b200.quant import codes_to, gemm

    g = torch.Generator(device=cuda).manual_seed(5)
    M, N, K, L = 600, 1024, 512, 300
    x = torch.randn(M, K, device=cuda, generator=g).bfloat16()
    q = _random_codes(fmt, N, K, cuda, 11)
    sc = torch.rand(N, device=cuda, generator=g) * 0.01
    wb = codes_to(q, fmt, torch.bfloat16)
    d = gemm(x, q, col_scale=sc, glu=True, codes=fmt)
    assert torch.equal(d.view(torch.int16), gemm(x, wb, col_scale=sc, glu=True).view(torch.int16))
    res = torch.randn(M, N, device=cuda, generator=g).bfloat16()
    gate = torch.randn(2, N, device=cuda, generator=g).bfloat16()
    o1, o2 = res.clone(), res.clone()
    gemm(x, q, col_scale=sc, gelu_col0=100, residual=o1, gate=gate, rows_per_gate=L, out=o1, codes=fmt)
    gemm(x, wb, col_scale=sc, gelu_col0=100, residual=o2, gate=gate, rows_per_gate=L, out=o2)
    assert torch.equal(o1.view(torch.int16), o2.view(torch.int16))


@pytest.mark.parametrize("fp8", [False, True])
@pytest.mark.parametrize("mn", [(64, 3072), (1, 18432), (128, 1000), (100, 64512), (64, 9216)])
def test_gemm_thin_tile_widths(cuda, mn, fp8):
    """Single-CTA products (M <= 128) over widths that select 64-, 128- and 256-column tiles
    (6 / 8-stage rings), ragged N, with bias, GELU on part of the columns and a gated
    residual, against fp64."""
    from quantfun2_b200.quant import gemm, quantize_rows

    M, N = mn
    K = 3072 if fp8 else 1024
    g = torch.Generator(device=cuda).manual_seed(N + M)
    x = torch.randn(M, K, device=cuda, generator=g).bfloat16()
    w = (torch.randn(N, K, device=cuda, generator=g) / K ** 0.5).bfloat16()
    bias = torch.randn(N, device=cuda, generator=g).bfloat16()
    res = torch.randn(M, N, device=cuda, generator=g).bfloat16()
    gate = torch.randn(1, N, device=cuda, generator=g).bfloat16()
    out = res.clone()
    if fp8:
        xq, xs = quantize_rows(x, "e4m3")
        wq, ws = quantize_rows(w, "e4m3")
        gemm(xq, wq, row_scale=xs, col_scale=ws, bias=bias, fp8=True, gelu_col0=N // 3, residual=out, gate=gate,
             rows_per_gate=M, out=out)
        xf = torch.from_numpy(e4m3_bits_to_f32(xq.cpu().numpy())).double().to(cuda) * xs.double()[:, None]
        wf = torch.from_numpy(e4m3_bits_to_f32(wq.cpu().numpy())).double().to(cuda) * ws.double()[:, None]
    else:
        gemm(x, w, bias=bias, gelu_col0=N // 3, residual=out, gate=gate, rows_per_gate=M, out=out)
        xf, wf = x.double(), w.double()
    y = xf @ wf.T + bias.double()
    y = torch.where(torch.arange(N, device=cuda) >= N // 3, torch.nn.functional.gelu(y, approximate="tanh"), y)
    ref = res.double() + gate.double() * y
    assert rel_err(out.float().cpu(), ref.cpu()) < 8e-3


@pytest.mark.parametrize("mnk", [(128, 256, 128), (300, 776, 272), (4608, 3072, 3072)])
def test_gemm_e4m3(cuda, mnk):
    from quantfun2_b200.quant import gemm, quantize_rows

    M, N, K = mnk
    g = torch.Generator(device=cuda).manual_seed(N)
    x = torch.randn(M, K, device=cuda, generator=g).bfloat16()
    w = torch.randn(N, K, device=cuda, generator=g).bfloat16()
    xq, xs = quantize_rows(x, "e4m3")
    wq, ws = quantize_rows(w, "e4m3")
    d = gemm(xq, wq, row_scale=xs, col_scale=ws, fp8=True, out_dtype=torch.float32)
    xf = torch.from_numpy(e4m3_bits_to_f32(xq.cpu().numpy())).double()
    wf = torch.from_numpy(e4m3_bits_to_f32(wq.cpu().numpy())).double()
    ref = (xf @ wf.T) * xs.cpu().double()[:, None] * ws.cpu().double()[None, :]
    assert rel_err(d.cpu(), ref) < 1e-5


@pytest.mark.parametrize("mode", ["int8", "fp8", "fp8_w8a8"])
@pytest.mark.parametrize("act", [torch.bfloat16, torch.float16])
def test_qlinear_vs_oracle_and_float(cuda, mode, act):
    from quantfun2_b200.quant import QLinear

    torch.manual_seed(1)
    lin = torch.nn.Linear(2304, 768, bias=True)
    x = torch.randn(4, 300, 2304).to(act)
    ql = QLinear.from_linear(lin.to(cuda).to(act), mode)
    y = ql(x.to(cuda))
    assert y.dtype == act
    y = y.float().cpu().numpy().reshape(-1, 768)
    codes = ql.codes.cpu().numpy()
    scale = ql.scale.cpu().numpy()
    bias = ql.bias.float().cpu().numpy()
    xs = x.float().numpy().reshape(-1, 2304)
    tag = "f16" if act == torch.float16 else "bf16"
    ref_q, ref_s = oq.quantize_weight_torchao(lin.weight.detach().to(act).float().cpu().numpy(),
                                              "int8" if mode == "int8" else "e4m3", tag)
    assert np.array_equal(codes.view(np.uint8), ref_q.view(np.uint8)) and np.array_equal(scale, ref_s)
    if mode == "fp8_w8a8":
        ref = oq.linear_w8a8_e4m3(xs, codes.view(np.uint8), scale, bias)
    else:
        ref = oq.linear_weight_only(xs, codes.view(np.uint8) if mode == "fp8" else codes, scale, bias,
                                    fp8=mode == "fp8")
    assert rel_err(y, ref) < 8e-3
    full = (xs.astype(np.float64) @ lin.weight.detach().to(act).float().cpu().numpy().astype(np.float64).T
            + lin.bias.detach().to(act).float().cpu().numpy())
    cos = float((y.ravel() @ full.ravel()) / math.sqrt((y.ravel() @ y.ravel()) * (full.ravel() @ full.ravel())))
    assert cos > (0.9999 if mode == "int8" else 0.999), cos


class _AttnLinears(torch.nn.Module):
    """The linears of the reference's JointAttention (src/models/common/attn.py:133-188):
    wq / wk / wv without bias, wo without bias, plus a biased MLP pair."""

    def __init__(self, dim=512, kv=256):
        super().__init__()
        self.wq = torch.nn.Linear(dim, dim, bias=False)
        self.wk = torch.nn.Linear(dim, kv, bias=False)
        self.wv = torch.nn.Linear(dim, kv, bias=False)
        self.wo = torch.nn.Linear(dim, dim, bias=False)
        self.mlp = torch.nn.Sequential(torch.nn.Linear(dim, 1024), torch.nn.SiLU(), torch.nn.Linear(1024, dim))

    def forward(self, x):
        return self.wo(self.wq(x)) + self.mlp(x) + self.wk(x).sum(-1, keepdim=True) * self.wv(x).mean()


@pytest.mark.parametrize("qname", ["qint8", "qfloat8"])
def test_quantize_model_keeps_modules_and_keys(cuda, qname):
    """quantize_model as the reference defines it (src/quant.py:131-148, :368-412): the
    nn.Linear modules stay, their weights become quantized tensor subclasses, the model
    ends in fp16 (the qdtype's activation dtype) and the state-dict keys do not change;
    F.linear on an fp16 activation runs the fp16 tcgen05 GEMM."""
    from quantfun2_b200 import quant

    torch.manual_seed(0)
    m = _AttnLinears()
    keys = list(m.state_dict().keys())
    wq0 = m.wq.weight.detach().half().float().numpy()
    x = torch.randn(3, 200, 512)
    ref = m(x).double()
    qm = quant.quantize_model(m, getattr(quant, qname), device="cuda", quantization_device="cuda")
    assert list(qm.state_dict().keys()) == keys
    for name in ["wq", "wk", "wv", "wo"]:
        lin = getattr(qm, name)
        assert type(lin) is torch.nn.Linear and isinstance(lin.weight, quant.QuantizedWeight)
        assert lin.weight.dtype == torch.float16 and lin.weight.shape == (lin.out_features, lin.in_features)
    assert qm.mlp[0].bias.dtype == torch.float16
    y = qm(x.to(cuda).half())
    assert y.dtype == torch.float16
    cos = torch.nn.functional.cosine_similarity(y.double().cpu().flatten(), ref.flatten(), dim=0).item()
    assert cos > (0.9999 if qname == "qint8" else 0.999), cos
    # the codes are torchao's, computed in fp16 arithmetic
    ref_q, ref_s = oq.quantize_weight_torchao(wq0, "int8" if qname == "qint8" else "e4m3", "f16")
    assert np.array_equal(qm.wq.weight.codes.cpu().numpy().view(np.uint8), ref_q.view(np.uint8))
    assert np.array_equal(qm.wq.weight.scale.cpu().numpy(), ref_s)


def test_gemm_fused_gelu_residual_gate(cuda):
    from quantfun2_b200.quant import gemm

    g = torch.Generator(device=cuda).manual_seed(3)
    M, N, K, L = 300, 512, 256, 150   # two "batches" of 150 rows for the gate
    a = torch.randn(M, K, device=cuda, generator=g).bfloat16()
    b = torch.randn(N, K, device=cuda, generator=g).bfloat16()
    res = torch.randn(M, N, device=cuda, generator=g).bfloat16()
    gate_full = torch.randn(2, 3 * N, device=cuda, generator=g).bfloat16()
    gate = gate_full[:, N:2 * N]                       # strided view, as the DiT blocks pass it
    y = (a.double() @ b.double().T)
    y = torch.where(torch.arange(N, device=cuda) >= 100, torch.nn.functional.gelu(y, approximate="tanh"), y)
    ref = res.double() + gate.double().repeat_interleave(L, 0) * y
    out = res.clone()
    gemm(a, b, gelu_col0=100, residual=out, gate=gate, rows_per_gate=L, out=out)   # in place
    assert rel_err(out.float().cpu(), ref.cpu()) < 8e-3


@pytest.mark.parametrize("fmt", ["bf16", "e4m3"])
def test_ln_modulate(cuda, fmt):
    from quantfun2_b200.quant import ln_modulate

    g = torch.Generator(device=cuda).manual_seed(4)
    B, L, N = 2, 100, 3072
    x = (torch.randn(B * L, N, device=cuda, generator=g) * 3 + 1).bfloat16()
    mod = torch.randn(B, 6 * N, device=cuda, generator=g).bfloat16()
    shift, scale = mod[:, N:2 * N], mod[:, 4 * N:5 * N]
    ref = torch.nn.functional.layer_norm(x.double(), (N,), eps=1e-6)
    ref = ref * (1 + scale.double().repeat_interleave(L, 0)) + shift.double().repeat_interleave(L, 0)
    out = ln_modulate(x, shift, scale, L, fmt)
    if fmt == "bf16":
        assert rel_err(out.float().cpu(), ref.cpu()) < 8e-3
    else:
        codes, s = out
        got = torch.from_numpy(e4m3_bits_to_f32(codes.cpu().numpy())) * s.cpu()[:, None]
        assert rel_err(got, ref.cpu()) < 0.07
        am = ref.abs().amax(1).cpu()
        assert torch.allclose(s.cpu().double(), am / 448, rtol=1e-3)
