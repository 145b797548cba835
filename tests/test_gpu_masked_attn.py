"""GPU: the attention processor seam (do_attn, mirror of src/models/common/attn.py:59-130)
on padded batches -- device-side unpad -> Sage varlen -> pad, no host sync -- and the bf16
tcgen05 attention of the flash / SDPA branches."""
import math

import pytest
import torch

pytestmark = pytest.mark.gpu


def _cos(a, b):
    return torch.nn.functional.cosine_similarity(a.double().flatten(), b.double().flatten(), dim=0).item()


def test_do_attn_padded_batch_matches_per_sequence_calls(cuda):
    from quantfun2_b200 import attention as A

    g = torch.Generator().manual_seed(3)
    B, S, Hq, Hkv, D = 3, 1100, 6, 2, 96
    q = torch.randn(B, S, Hq, D, generator=g).bfloat16().to(cuda)
    k = (torch.randn(B, S, Hkv, D, generator=g) + 2 * torch.randn(1, 1, Hkv, D, generator=g)).bfloat16().to(cuda)
    v = torch.randn(B, S, Hkv, D, generator=g).bfloat16().to(cuda)
    mask = torch.ones(B, S, dtype=torch.bool)
    mask[1, 700:] = False                                   # padded tail
    mask[2] = torch.rand(S, generator=g) < 0.6              # holes anywhere
    mask = mask.to(cuda)
    A.ATTN = "b200"
    out = A.do_attn(None, q, k, v, mask)
    assert out.shape == q.shape
    for b in range(B):
        sel = mask[b]
        n = int(sel.sum())
        cu = torch.tensor([0, n], dtype=torch.int32, device=cuda)
        # the same sequence alone through the varlen entry (a dense call on few heads may
        # split the K/V tiles across CTAs, which rounds P differently by design)
        ref = A.sageattn_varlen(q[b, sel], k[b, sel], v[b, sel], cu, cu, n, n)
        assert torch.equal(out[b, sel], ref), b                    # same per-sequence kernel math
        assert not out[b, ~sel].any()                                # padded rows are zero
        kk = k[b:b + 1, sel].repeat_interleave(Hq // Hkv, 2)
        vv = v[b:b + 1, sel].repeat_interleave(Hq // Hkv, 2)
        exact = torch.nn.functional.scaled_dot_product_attention(
            q[b:b + 1, sel].transpose(1, 2).float(), kk.transpose(1, 2).float(), vv.transpose(1, 2).float())
        assert _cos(out[b:b + 1, sel].transpose(1, 2), exact) >= 0.998
        dense = A.sageattn(q[b:b + 1, sel], k[b:b + 1, sel], v[b:b + 1, sel], tensor_layout="NHD")
        assert _cos(dense, out[b:b + 1, sel]) >= 0.9995


def test_flash_branch_bf16_dense(cuda):
    from quantfun2_b200 import attention as A

    g = torch.Generator().manual_seed(4)
    B, S, H, D = 2, 1000, 4, 128
    q, k, v = (torch.randn(B, S, H, D, generator=g).bfloat16().to(cuda) for _ in range(3))
    A.ATTN = "flash"
    try:
        out = A.do_attn(None, q, k, v, None)
        with pytest.raises(A.QF2Error):
            A.do_attn(None, q, k, v, torch.ones(B, S, dtype=torch.bool, device=cuda))
    finally:
        A.ATTN = "b200"
    exact = torch.nn.functional.scaled_dot_product_attention(q.transpose(1, 2).float(), k.transpose(1, 2).float(),
                                                             v.transpose(1, 2).float()).transpose(1, 2)
    c = _cos(out, exact)
    print(f"flash branch cos={c:.6f} maxabs={(out.float() - exact).abs().max().item():.4g}")
    assert c >= 0.9999
