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
def test_qlinear_vs_oracle_and_float(cuda, mode):
    from quantfun2_b200.quant import QLinear

    torch.manual_seed(1)
    lin = torch.nn.Linear(2304, 768, bias=True)
    x = torch.randn(4, 300, 2304).bfloat16()
    ql = QLinear.from_linear(lin.to(cuda).bfloat16(), mode)
    y = ql(x.to(cuda)).float().cpu().numpy().reshape(-1, 768)
    codes = ql.codes.cpu().numpy()
    scale = ql.scale.cpu().numpy()
    bias = ql.bias.float().cpu().numpy()
    xs = x.float().numpy().reshape(-1, 2304)
    if mode == "fp8_w8a8":
        ref = oq.linear_w8a8_e4m3(xs, codes.view(np.uint8), scale, bias)
    else:
        ref = oq.linear_weight_only(xs, codes.view(np.uint8) if mode == "fp8" else codes, scale, bias,
                                    fp8=mode == "fp8")
    assert rel_err(y, ref) < 8e-3
    full = (xs.astype(np.float64) @ lin.weight.detach().bfloat16().float().cpu().numpy().astype(np.float64).T
            + lin.bias.detach().bfloat16().float().cpu().numpy())
    cos = float((y.ravel() @ full.ravel()) / math.sqrt((y.ravel() @ y.ravel()) * (full.ravel() @ full.ravel())))
    assert cos > (0.9999 if mode == "int8" else 0.999), cos


def test_quantize_model_swaps_linears(cuda):
    from quantfun2_b200.quant import QLinear, qint8, quantize_model

    torch.manual_seed(0)
    m = torch.nn.Sequential(torch.nn.Linear(256, 512), torch.nn.SiLU(), torch.nn.Linear(512, 256))
    x = torch.randn(64, 256)
    ref = m(x)
    qm = quantize_model(m, qint8, device="cuda", quantization_device="cuda")
    assert isinstance(qm[0], QLinear) and isinstance(qm[2], QLinear)
    y = qm(x.to(cuda).bfloat16()).float().cpu()
    cos = torch.nn.functional.cosine_similarity(y.flatten(), ref.flatten(), dim=0).item()
    assert cos > 0.999


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
