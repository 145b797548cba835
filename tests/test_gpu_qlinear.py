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
