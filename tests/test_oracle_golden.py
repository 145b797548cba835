"""CPU: pin the oracle restatements to golden vectors produced by the reference code
(tests/golden/make_golden.py imports the reference's eager bodies)."""
import math

import numpy as np
import pytest

from oracle import ops, sage
from tests.golden_cases import jattn_case
from oracle.numerics import bf16_bits_to_f32, f32_to_bf16_bits, round_bf16


def cplx(a):
    return a[..., 0] + 1j * a[..., 1]


def test_rope_f32_matches_reference(golden):
    f = cplx(golden["rope_freqs"]).astype(np.complex64)
    oq, ok = ops.rope_apply(golden["rope_f32_xq"], golden["rope_f32_xk"], f, "f32")
    np.testing.assert_allclose(oq, golden["rope_f32_oq"], rtol=0, atol=2e-6)
    np.testing.assert_allclose(ok, golden["rope_f32_ok"], rtol=0, atol=2e-6)


def test_rope_bf16_matches_reference_bits(golden):
    f = cplx(golden["rope_freqs"]).astype(np.complex64)
    xq = bf16_bits_to_f32(golden["rope_bf16_xq"])
    xk = bf16_bits_to_f32(golden["rope_bf16_xk"])
    oq, ok = ops.rope_apply(xq, xk, f, "bf16")
    for got, ref in ((oq, golden["rope_bf16_oq"]), (ok, golden["rope_bf16_ok"])):
        gb = f32_to_bf16_bits(got).astype(np.int32)
        diff = np.abs(gb - ref.astype(np.int32))
        assert diff.max() <= 1, diff.max()          # at most one bf16 ulp
        assert (diff == 0).mean() > 0.999


@pytest.mark.parametrize("tag", ["head", "row"])
def test_rmsnorm_matches_reference(golden, tag):
    eps = float(golden[f"rms_{tag}_eps"][0])
    y = ops.rmsnorm_apply(golden[f"rms_{tag}_x_f32"], golden[f"rms_{tag}_w_f32"], eps, "f32")
    np.testing.assert_allclose(y, golden[f"rms_{tag}_y_f32"], rtol=2e-6, atol=2e-6)
    xb = bf16_bits_to_f32(golden[f"rms_{tag}_x_bf16"])
    wb = bf16_bits_to_f32(golden[f"rms_{tag}_w_bf16"])
    yb = ops.rmsnorm_apply(xb, wb, eps, "bf16")
    diff = np.abs(f32_to_bf16_bits(yb).astype(np.int32) - golden[f"rms_{tag}_y_bf16"].astype(np.int32))
    assert diff.max() <= 1 and (diff == 0).mean() > 0.99


def test_softmax_matches_reference(golden):
    y = ops.softmax_lastdim(golden["softmax_x_f32"], "f32")
    np.testing.assert_allclose(y, golden["softmax_y_f32"], rtol=1e-5, atol=1e-7)
    yb = ops.softmax_lastdim(bf16_bits_to_f32(golden["softmax_x_bf16"]), "bf16")
    diff = np.abs(f32_to_bf16_bits(yb).astype(np.int32) - golden["softmax_y_bf16"].astype(np.int32))
    assert diff.max() <= 1


def _joint_attention_oracle(g):
    dim, heads, kvh, seq = [int(v) for v in g["jattn_meta"]]
    D = dim // heads
    x = g["jattn_x"].astype(np.float64)[0]
    q = (x @ g["jattn_wq"].T.astype(np.float64)).astype(np.float32).reshape(1, seq, heads, D)
    k = (x @ g["jattn_wk"].T.astype(np.float64)).astype(np.float32).reshape(1, seq, kvh, D)
    v = (x @ g["jattn_wv"].T.astype(np.float64)).astype(np.float32).reshape(1, seq, kvh, D)
    q = ops.rmsnorm_apply(q, g["jattn_qnorm"], 1e-6, "f32")
    k = ops.rmsnorm_apply(k, g["jattn_knorm"], 1e-6, "f32")
    f = cplx(g["jattn_freqs"]).astype(np.complex64)
    q, k = ops.rope_apply(q, k, f, "f32")
    o = sage.sdpa_reference(q.transpose(0, 2, 1, 3), k.transpose(0, 2, 1, 3), v.transpose(0, 2, 1, 3),
                            1.0 / math.sqrt(D))
    o = o.transpose(0, 2, 1, 3).reshape(1, seq, dim)
    return (o.astype(np.float64) @ g["jattn_wo"].T.astype(np.float64)).astype(np.float32)


def test_joint_attention_block_composition(golden):
    """The oracle's QKV -> per-head RMSNorm -> RoPE -> SDPA -> O composition reproduces
    the reference JointAttention.forward (src/models/common/attn.py:190-236)."""
    y = _joint_attention_oracle(golden)
    np.testing.assert_allclose(y, golden["jattn_y"], rtol=1e-4, atol=1e-5)


def test_sage_oracle_close_to_sdpa():
    rng = np.random.default_rng(0)
    B, H, S, D = 1, 2, 200, 128
    q = round_bf16(rng.standard_normal((B, H, S, D)).astype(np.float32))
    k = round_bf16((rng.standard_normal((B, H, S, D)) + 3 * rng.standard_normal((1, H, 1, D))).astype(np.float32))
    v = round_bf16(rng.standard_normal((B, H, S, D)).astype(np.float32))
    o = sage.sageattn(q, k, v)
    r = sage.sdpa_reference(q, k, v)
    cos = float((o * r).sum() / np.sqrt((o * o).sum() * (r * r).sum()))
    assert cos > 0.995, cos


def test_sage_quant_rules():
    """Hand-checkable cases of the published rule (x / scale, + 0.5 * sign, truncate)."""
    x = np.zeros((64, 128), np.float32)
    x[0, 0], x[1, 1], x[2, 2], x[3, 3] = 127.0, 63.5, -0.5, 2.5   # scale 1.0: halves go away from zero
    x[4, 4] = np.nextafter(np.float32(0.5), np.float32(0))         # 0.5 - 2^-25: the fp32 add rounds to 1.0
    x[5, 5] = np.float32(-2.4999998)
    codes, scales = sage._block_quant(x)
    assert scales[0] == np.float32(1.0)
    assert codes[0, 0] == 127 and codes[1, 1] == 64 and codes[2, 2] == -1 and codes[3, 3] == 3
    assert codes[4, 4] == 1 and codes[5, 5] == -2
    z, zs = sage._block_quant(np.zeros((70, 128), np.float32))
    assert (z == 0).all() and (zs == 1.0).all() and zs.shape == (2,)


def test_torchao_weight_rule_cases():
    """Hand-checkable cases of the torchao 0.7.0 weight rule in fp16."""
    from oracle import qlinear as oq

    w = np.zeros((3, 4), np.float32)
    w[0] = [1.0, -0.5, 0.25, 0.0]        # scale = f16(1/127.5); codes round half to even in fp16
    w[2] = [1e-4, -1e-4, 0.0, 5e-5]      # fp16 scale ~7.8e-7: 1/scale overflows fp16 -> inf
    q, s = oq.quantize_weight_torchao(w, "int8", "f16")
    assert s[0] == np.float32(np.float16(np.float32(1.0) / np.float32(127.5)))
    assert q[0, 0] == 127 and q[0, 3] == 0
    assert s[1] == np.float32(np.finfo(np.float32).eps) and (q[1] == 0).all()   # zero row: clamp to eps
    assert q[2, 0] == 127 and q[2, 1] == -128 and q[2, 2] == 0                   # inf * 0 = nan -> 0
    q8, s8 = oq.quantize_weight_torchao(w, "e4m3", "f16")
    assert q8[0, 0] == 0x7E   # 448


@pytest.mark.parametrize("tag", ["d128", "d96"])
def test_joint_attention_golden_head_dims(tag):
    """The oracle composition reproduces the reference JointAttention at head dims 128 and
    96 with GQA and a ragged last tile (tests/golden/ref_jattn.npz)."""
    c = jattn_case(tag)
    D = c["dim"] // c["heads"]
    x = c["x"][0].astype(np.float64)
    w = c["w"]
    q = (x @ w["wq"].T.astype(np.float64)).astype(np.float32).reshape(1, c["seq"], c["heads"], D)
    k = (x @ w["wk"].T.astype(np.float64)).astype(np.float32).reshape(1, c["seq"], c["kvh"], D)
    v = (x @ w["wv"].T.astype(np.float64)).astype(np.float32).reshape(1, c["seq"], c["kvh"], D)
    q = ops.rmsnorm_apply(q, w["q_norm"], 1e-6, "f32")
    k = ops.rmsnorm_apply(k, w["k_norm"], 1e-6, "f32")
    q, k = ops.rope_apply(q, k, cplx(c["freqs"]).astype(np.complex64), "f32")
    o = sage.sdpa_reference(q.transpose(0, 2, 1, 3), k.transpose(0, 2, 1, 3), v.transpose(0, 2, 1, 3),
                            1.0 / math.sqrt(D))
    y = (o.transpose(0, 2, 1, 3).reshape(1, c["seq"], c["dim"]).astype(np.float64)
         @ w["wo"].T.astype(np.float64)).astype(np.float32)
    np.testing.assert_allclose(y, c["y"], rtol=1e-4, atol=2e-5)
