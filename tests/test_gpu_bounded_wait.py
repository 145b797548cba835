"""GPU: failure detection of the attention kernel's bounded waits, without a GPU fault.

qf2_sage_fault_injection shortens every mbarrier wait of the attention kernel to ~2 ms and
makes its producer leave one K/V tile unloaded -- a barrier nothing completes.  The MMA
and softmax warps waiting on it give up, the kernel records a timeout in the workspace
status word, lets its issued copies land, drains its MMAs, frees TMEM and returns.  The
host reads QF2_ERR_TIMEOUT, and the next normal call on the same context is correct.
"""
import math

import numpy as np
import pytest
import torch

from oracle import sage
from quantfun2_b200 import _lib
from quantfun2_b200._lib import i64, stream_ptr

pytestmark = pytest.mark.gpu

QF2_ERR_TIMEOUT = -4


def _qkv(dev, B, H, S, seed):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, H, S, 128, generator=g).bfloat16()
    k = (torch.randn(B, H, S, 128, generator=g) + 3 * torch.randn(1, H, 1, 128, generator=g)).bfloat16()
    v = torch.randn(B, H, S, 128, generator=g).bfloat16()
    return q, k, v


def _call(lib, q, k, v, out, ws):
    st = lambda t: i64(t.stride(0), t.stride(1), t.stride(2))  # noqa: E731
    B, H, S, D = q.shape
    return lib.qf2_sageattn(q.data_ptr(), st(q), k.data_ptr(), st(k), v.data_ptr(), st(v), out.data_ptr(), st(out),
                            B, H, H, S, S, D, 1.0 / math.sqrt(D), _lib.QF2_BF16, ws.data_ptr(), ws.numel(),
                            stream_ptr(q.device))


def test_attention_wait_times_out_then_recovers(cuda):
    from quantfun2_b200.attention import _workspace

    lib = _lib.load()
    B, H, S = 1, 2, 1024
    qc, kc, vc = _qkv(cuda, B, H, S, 21)
    q, k, v = qc.to(cuda), kc.to(cuda), vc.to(cuda)
    out = torch.zeros_like(q)
    ws = _workspace(int(lib.qf2_sage_workspace_bytes(B, H, H, B * S, B * S, S, S, 128)), cuda)
    assert _call(lib, q, k, v, out, ws) == 0               # a clean call first
    assert lib.qf2_workspace_status(ws.data_ptr(), stream_ptr(cuda)) == 0
    clean = out.clone()
    assert lib.qf2_sage_fault_injection(2000, 3) == 0
    try:
        out.zero_()
        assert _call(lib, q, k, v, out, ws) == 0            # launched fine
        assert lib.qf2_workspace_status(ws.data_ptr(), stream_ptr(cuda)) == QF2_ERR_TIMEOUT
        assert lib.qf2_workspace_status(ws.data_ptr(), stream_ptr(cuda)) == 0   # read clears it
    finally:
        lib.qf2_sage_fault_injection(0, -1)
    # the context is intact: a normal call on it gives the clean call's output bit for bit
    assert _call(lib, q, k, v, out, ws) == 0
    assert lib.qf2_workspace_status(ws.data_ptr(), stream_ptr(cuda)) == 0
    assert torch.equal(out, clean)
    o = out.float().cpu().numpy()
    ref = sage.sageattn(qc.float().numpy(), kc.float().numpy(), vc.float().numpy())
    cos = float((o * ref).sum() / np.sqrt((o * o).sum() * (ref * ref).sum()))
    assert cos >= 0.999, cos
