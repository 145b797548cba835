"""GPU parity of top-k block-sparse attention: kept block indices bit-exact against the
oracle; attention output within bf16 tolerance of the fp64 oracle."""
import math

import numpy as np
import pytest
import torch

from oracle import blocktopk as bt

pytestmark = pytest.mark.gpu


def cosine(a, b):
    a = a.astype(np.float64).ravel()
    b = b.astype(np.float64).ravel()
    return float(a @ b / math.sqrt((a @ a) * (b @ b)))


def bf16_inputs(B, Hq, Hkv, S, seed, hot=True):
    if hot:
        q, k, v = bt.make_hot_inputs(B, Hq, S, 128, hot=4, boost=2.0, seed=seed)
        k, v = k[:, :Hkv], v[:, :Hkv]
    else:
        rng = np.random.default_rng(seed)
        q = rng.standard_normal((B, Hq, S, 128), dtype=np.float32)
        k = rng.standard_normal((B, Hkv, S, 128), dtype=np.float32)
        v = rng.standard_normal((B, Hkv, S, 128), dtype=np.float32)
    t = [torch.from_numpy(np.ascontiguousarray(x)).bfloat16() for x in (q, k, v)]
    return t, [x.float().numpy() for x in t]


@pytest.mark.parametrize("shape", [(1, 2, 2, 1000, 3), (2, 4, 2, 777, 2), (1, 2, 1, 256, 2)])
def test_select_indices_bit_exact(cuda, shape):
    from quantfun2_b200.attention import block_topk_select

    B, Hq, Hkv, S, keep = shape
    (q, k, v), (qn, kn, vn) = bf16_inputs(B, Hq, Hkv, S, seed=S)
    idx = block_topk_select(q.to(cuda), k.to(cuda), keep).cpu().numpy()
    for b in range(B):
        for h in range(Hq):
            ref = bt.select_head(qn[b, h], kn[b, h // (Hq // Hkv)], keep)
            assert np.array_equal(idx[b, h], ref), (b, h)


@pytest.mark.parametrize("shape", [(1, 2, 2, 1000, 3), (2, 4, 2, 777, 7), (1, 2, 1, 384, 3), (1, 2, 2, 1000, 1),
                                   (2, 2, 1, 300, 2)])
@pytest.mark.parametrize("layout", ["HND", "NHD"])
def test_blocksparse_attention_vs_oracle(cuda, shape, layout):
    from quantfun2_b200.attention import block_topk_select, blocksparse_attn

    B, Hq, Hkv, S, keep = shape
    (q, k, v), (qn, kn, vn) = bf16_inputs(B, Hq, Hkv, S, seed=7)
    tr = (lambda t: t) if layout == "HND" else (lambda t: t.transpose(1, 2).contiguous())
    qd, kd, vd = tr(q).to(cuda), tr(k).to(cuda), tr(v).to(cuda)
    idx = block_topk_select(qd, kd, keep, tensor_layout=layout)
    o = blocksparse_attn(qd, kd, vd, idx, tensor_layout=layout)
    if layout == "NHD":
        o = o.transpose(1, 2)
    o = o.float().cpu().numpy()
    ref = np.zeros_like(o)
    idn = idx.cpu().numpy()
    for b in range(B):
        for h in range(Hq):
            hk = h // (Hq // Hkv)
            ref[b, h] = bt.attention_head(qn[b, h], kn[b, hk], vn[b, hk], idn[b, h], 1 / math.sqrt(128))
    c = cosine(o, ref)
    err = np.abs(o - ref).max()
    print(f"cos={c:.7f} maxabs={err:.4g}")
    assert c >= 0.9999 and err < 0.03


def test_keep_all_blocks_matches_dense_sdpa(cuda):
    from quantfun2_b200.attention import blocksparse_attn

    (q, k, v), _ = bf16_inputs(1, 3, 3, 640, seed=2, hot=False)
    q, k, v = q.to(cuda), k.to(cuda), v.to(cuda)
    idx = torch.arange(5, dtype=torch.int32, device=cuda).expand(1, 3, 5, 5).contiguous()
    o = blocksparse_attn(q, k, v, idx).float()
    r = torch.nn.functional.scaled_dot_product_attention(q.float(), k.float(), v.float())
    c = torch.nn.functional.cosine_similarity(o.flatten(), r.flatten(), dim=0).item()
    assert c >= 0.9999 and (o - r).abs().max().item() < 0.02


def test_topk_attn_dropin_and_pos_dict_reuse(cuda):
    from quantfun2_b200.kernels import topk_attn

    (q, k, v), (qn, kn, vn) = bf16_inputs(1, 4, 2, 512, seed=4)
    xq, xk, xv = (t.transpose(1, 2).contiguous().to(cuda) for t in (q, k, v))  # [B, S, H, D]
    out, pos = topk_attn(xq, xk, xv, None, None, 128, TOP_K=256, POS_DICT=None, N_HEADS=4, N_KV_HEADS=2)
    assert out.shape == xq.shape and pos.shape == (1, 4, 4, 2)
    out2, pos2 = topk_attn(xq, xk, xv, None, None, 128, TOP_K=256, POS_DICT=pos, N_HEADS=4, N_KV_HEADS=2)
    assert pos2 is pos and torch.equal(out, out2)


def test_flux_16k_shape_indices_and_spot_rows(cuda):
    """The benchmarked shape (16384 tokens, 12.5% of blocks kept) on two heads: all
    indices bit-exact, and four query blocks checked against the fp64 oracle."""
    from quantfun2_b200.attention import block_topk_select, blocksparse_attn

    S, H, keep = 16384, 2, 16
    (q, k, v), (qn, kn, vn) = bf16_inputs(1, H, H, S, seed=11)
    qd, kd, vd = q.to(cuda), k.to(cuda), v.to(cuda)
    idx = block_topk_select(qd, kd, keep)
    o = blocksparse_attn(qd, kd, vd, idx).float().cpu().numpy()
    idn = idx.cpu().numpy()
    for h in range(H):
        assert np.array_equal(idn[0, h], bt.select_head(qn[0, h], kn[0, h], keep)), h
        for qb in (0, 17, 64, 127):
            sub = bt.attention_head(qn[0, h, qb * 128:(qb + 1) * 128], kn[0, h], vn[0, h], idn[0, h, qb:qb + 1],
                                    1 / math.sqrt(128))
            got = o[0, h, qb * 128:(qb + 1) * 128]
            assert cosine(got, sub) >= 0.9999 and np.abs(got - sub).max() < 0.03, (h, qb)
