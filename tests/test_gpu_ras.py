"""GPU: the RAS partial ops of the reference (region-adaptive sampling: only the active
token rows are recomputed and scattered into the full sequence).

  rope_scatter      PYCUDA_ROPE_KERNEL (src/kernels/cuda/ras.cu:12-52): bit-exact against
                    the oracle's stated rounding, untouched rows kept, bad index reported
  partially_linear  _partially_linear (src/kernels/triton/ras.py:28-128) on the tcgen05
                    GEMM with a row-scatter epilogue: within bf16 rounding of fp64
"""
import numpy as np
import pytest
import torch

from oracle import ops
from oracle.numerics import round_bf16

pytestmark = pytest.mark.gpu


def _bits(t):
    return t.contiguous().view(torch.int16).cpu().numpy()


@pytest.mark.parametrize("B,N,M,H,D", [(2, 300, 512, 24, 128), (1, 77, 77, 3, 96)])
def test_rope_scatter_bit_exact(cuda, B, N, M, H, D):
    from quantfun2_b200.kernels import rope_scatter

    g = torch.Generator().manual_seed(N)
    x = torch.randn(B, N, H, D, generator=g).bfloat16()
    ang = torch.rand(N, D // 2, generator=g) * 6.3
    f = torch.stack([torch.cos(ang), torch.sin(ang)], -1).reshape(N, D).float()
    idx = torch.randperm(M, generator=g)[:N]
    y0 = torch.full((B, M, H, D), 7.0).bfloat16()
    y = rope_scatter(x.to(cuda), f[None].to(cuda), idx.to(cuda), y0.clone().to(cuda))
    ref = ops.rope_scatter(x.float().numpy(), f.numpy(), idx.numpy(), y0.float().numpy())
    got = y.float().cpu().numpy()
    assert np.array_equal(got, ref)
    rest = np.setdiff1d(np.arange(M), idx.numpy())
    assert (got[:, rest] == 7.0).all()


def test_rope_scatter_rejects_bad_index(cuda):
    from quantfun2_b200._lib import QF2Error
    from quantfun2_b200.kernels import rope_scatter

    x = torch.randn(1, 4, 2, 64, device=cuda).bfloat16()
    f = torch.ones(4, 64, device=cuda)
    y = torch.zeros(1, 8, 2, 64, device=cuda).bfloat16()
    with pytest.raises(QF2Error, match="index range"):
        rope_scatter(x, f, torch.tensor([0, 9, 2, 3], device=cuda), y)
    assert not y[:, 1].any() and y[:, 0].any()      # the bad row is skipped, the others written


@pytest.mark.parametrize("B,M,K,N,M_out", [(2, 300, 512, 512, 300), (1, 1000, 3072, 3072, 4608), (3, 64, 256, 384, 80)])
def test_partially_linear_scatter(cuda, B, M, K, N, M_out):
    from quantfun2_b200.kernels import partially_linear

    g = torch.Generator().manual_seed(M + K)
    x = torch.randn(B, M, K, generator=g).bfloat16()
    w = (torch.randn(N, K, generator=g) / K ** 0.5).bfloat16()
    idx = torch.randperm(M_out, generator=g)[:M]
    out0 = torch.full((B, M_out, N), -3.0).bfloat16()
    got = partially_linear(x.to(cuda), w.to(cuda), idx.to(cuda), out=out0.clone().to(cuda)).float().cpu().numpy()
    ref = ops.partially_linear(x.float().numpy(), w.float().numpy(), idx.numpy(), out0.float().numpy())
    rows = idx.numpy()
    err = np.abs(got[:, rows] - ref[:, rows])
    assert (err <= 2 ** -7 * np.abs(ref[:, rows]) + 1e-3).all(), err.max()   # one bf16 rounding
    rest = np.setdiff1d(np.arange(M_out), rows)
    assert (got[:, rest] == -3.0).all()
    # without `out`: a new [B, M, N] tensor, every row named once by a permutation of M
    perm = torch.randperm(M, generator=g)
    y = partially_linear(x.to(cuda), w.to(cuda), perm.to(cuda)).float().cpu().numpy()
    full = np.einsum("bmk,nk->bmn", x.double().numpy(), w.double().numpy())
    assert np.allclose(y[:, perm.numpy()], full, rtol=2 ** -7, atol=1e-3)
