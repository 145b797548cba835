"""GPU: the B200 attention block on the reference's own JointAttention outputs.

tests/golden/ref_jattn.npz holds JointAttention.forward (src/models/common/attn.py:190-236)
of the reference, run by tests/golden/make_golden.py on the CPU in fp32 through its SDPA
branch (GQA, a ragged last 128-token tile).  Here the same inputs and weights (bf16
values) go through the sm_100a path: bf16 tcgen05 GEMM for the fused QKV projection ->
fused per-head RMSNorm + RoPE -> Sage INT8/FP8 attention -> bf16 GEMM for the output
projection.  Tolerance: cosine >= 0.999 against the reference output; max-abs reported.
"""
import math

import numpy as np
import pytest
import torch

from tests.golden_cases import jattn_case

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("tag", ["d128", "d96"])
def test_b200_joint_attention_block_vs_reference_golden(cuda, tag):
    from quantfun2_b200.attention import sageattn
    from quantfun2_b200.kernels import qkv_norm_rope
    from quantfun2_b200.quant import gemm

    c = jattn_case(tag)
    H, Hkv, seq, dim = c["heads"], c["kvh"], c["seq"], c["dim"]
    D = dim // H
    w = {k: torch.from_numpy(v).to(cuda) for k, v in c["w"].items()}
    x = torch.from_numpy(c["x"][0]).to(cuda).bfloat16()                       # [seq, dim]
    wqkv = torch.cat([w["wq"], w["wk"], w["wv"]]).bfloat16()
    qkv = gemm(x, wqkv).view(1, seq, -1)
    q = torch.empty(1, seq, H, D, device=cuda, dtype=torch.bfloat16)
    k = torch.empty(1, seq, Hkv, D, device=cuda, dtype=torch.bfloat16)
    v = torch.empty_like(k)
    freqs = torch.view_as_complex(torch.from_numpy(c["freqs"]).contiguous()).to(cuda)
    qkv_norm_rope(qkv, H, w["q_norm"].bfloat16(), w["k_norm"].bfloat16(), freqs, q, k, v, eps=1e-6, Hkv=Hkv)
    o = sageattn(q, k, v, tensor_layout="NHD", sm_scale=1.0 / math.sqrt(D))
    y = gemm(o.reshape(seq, dim), w["wo"].bfloat16(), out_dtype=torch.float32)
    torch.cuda.synchronize()
    got = y.cpu().double().numpy()
    ref = c["y"][0].astype(np.float64)
    cos = float(got.ravel() @ ref.ravel() / math.sqrt((got.ravel() @ got.ravel()) * (ref.ravel() @ ref.ravel())))
    err = float(np.abs(got - ref).max())
    print(f"{tag}: cos={cos:.6f} maxabs={err:.4g} (|ref|max={np.abs(ref).max():.3g})")
    assert cos >= 0.999, cos
    assert err < 0.05 * np.abs(ref).max()
