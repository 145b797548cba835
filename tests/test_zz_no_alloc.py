"""qf2_sageattn_noalloc: Sage attention for callers that cannot allocate device memory.

Such callers (a host program that keeps all device memory in its own pool, code that
must not trigger an allocation's device synchronization, a binding that only holds the
tensors it passes) get the quantization scratch from a static device array inside the
library instead of a workspace argument.  This file is collected last so that a
failure here comes after every other test has run; it passes alone or after them.
"""
import math

import pytest
import torch

from quantfun2_b200 import _lib
from quantfun2_b200._lib import i64, stream_ptr

pytestmark = pytest.mark.gpu

QF2_ERR_WORKSPACE = -6
QF2_ERR_TIMEOUT = -4


def _inputs(dev, B, Hq, Hkv, S, seed, dtype=torch.bfloat16):
    g = torch.Generator(device=dev).manual_seed(seed)
    q = torch.randn(B, Hq, S, 128, device=dev, generator=g).to(dtype)
    k = (torch.randn(B, Hkv, S, 128, device=dev, generator=g)
         + 3.0 * torch.randn(1, Hkv, 1, 128, device=dev, generator=g)).to(dtype)
    v = torch.randn(B, Hkv, S, 128, device=dev, generator=g).to(dtype)
    return q, k, v


def _strides(t):
    return i64(t.stride(0), t.stride(1), t.stride(2))


def _dt(t):
    return _lib.QF2_BF16 if t.dtype == torch.bfloat16 else _lib.QF2_F16


def _with_workspace(lib, q, k, v, sm):
    """The existing entry point, with a caller-provided workspace."""
    B, Hq, S, D = q.shape
    Hkv = k.shape[1]
    out = torch.empty_like(q)
    nbytes = int(lib.qf2_sage_workspace_bytes(B, Hq, Hkv, B * S, B * S, S, S, D))
    raw = torch.empty(nbytes + 1024, dtype=torch.uint8, device=q.device)
    ws = raw[(-raw.data_ptr()) % 1024:][:nbytes]
    st = lib.qf2_sageattn(q.data_ptr(), _strides(q), k.data_ptr(), _strides(k), v.data_ptr(), _strides(v),
                          out.data_ptr(), _strides(out), B, Hq, Hkv, S, S, D, sm, _dt(q), ws.data_ptr(), nbytes,
                          stream_ptr(q.device))
    assert st == 0, lib.qf2_status_string(st)
    return out


def _noalloc(lib, q, k, v, sm):
    B, Hq, S, D = q.shape
    Hkv = k.shape[1]
    out = torch.empty_like(q)
    st = lib.qf2_sageattn_noalloc(q.data_ptr(), _strides(q), k.data_ptr(), _strides(k), v.data_ptr(), _strides(v),
                                  out.data_ptr(), _strides(out), B, Hq, Hkv, S, S, D, sm, _dt(q),
                                  stream_ptr(q.device))
    assert st == 0, lib.qf2_status_string(st)
    return out


@pytest.mark.parametrize("B,Hq,Hkv,S,seed,dtype", [
    (1, 24, 24, 4608, 1, torch.bfloat16),   # one Flux-shaped sequence
    (2, 3, 3, 777, 2, torch.bfloat16),      # ragged length
    (1, 4, 4, 1000, 3, torch.float16),      # fp16 inputs
    (2, 6, 2, 777, 4, torch.bfloat16),      # GQA: 3 query heads per kv head
])
def test_noalloc_matches_workspace_entry_point_twice(cuda, B, Hq, Hkv, S, seed, dtype):
    lib = _lib.load()
    sm = 1.0 / math.sqrt(128)
    q, k, v = _inputs(cuda, B, Hq, Hkv, S, seed, dtype)
    # two calls in a row: the second runs over the first call's leftovers in the shared
    # static array (and over the previous case's, when the cases run in one process)
    for _ in range(2):
        got = _noalloc(lib, q, k, v, sm)
        assert lib.qf2_sageattn_noalloc_status(stream_ptr(cuda)) == 0   # no bounded wait gave up
        ref = _with_workspace(lib, q, k, v, sm)
        torch.cuda.synchronize()
        assert torch.isfinite(got).all()
        # same kernels, same arithmetic: identical up to the tolerance the Sage tests use
        cos = torch.nn.functional.cosine_similarity(got.float().flatten(), ref.float().flatten(), dim=0).item()
        assert cos >= 0.9995, cos
        assert (got.float() - ref.float()).abs().max().item() <= 1e-2
        assert torch.equal(got, ref)


def test_noalloc_rejects_problems_beyond_its_scratch(cuda):
    lib = _lib.load()
    q, k, v = _inputs(cuda, 2, 24, 24, 4608, 3)   # ~85 MB of codes: more than the 48 MiB array
    out = torch.zeros_like(q)
    st = lib.qf2_sageattn_noalloc(q.data_ptr(), _strides(q), k.data_ptr(), _strides(k), v.data_ptr(), _strides(v),
                                  out.data_ptr(), _strides(out), 2, 24, 24, 4608, 4608, 128, 0.088, _lib.QF2_BF16,
                                  stream_ptr(cuda))
    assert st == QF2_ERR_WORKSPACE
    torch.cuda.synchronize()
    assert not out.any()   # nothing was launched


def test_noalloc_status_reports_a_timed_out_call(cuda):
    """A caller without a workspace pointer still learns that a bounded device wait gave
    up: the test makes one (qf2_sage_fault_injection: ~2 ms waits, one K/V load never
    issued), qf2_sageattn_noalloc_status reports it once and clears it, and the next
    normal call matches the workspace entry point again."""
    lib = _lib.load()
    sm = 1.0 / math.sqrt(128)
    q, k, v = _inputs(cuda, 1, 2, 2, 1024, 7)
    assert lib.qf2_sage_fault_injection(2000, 2) == 0
    try:
        _noalloc(lib, q, k, v, sm)
        assert lib.qf2_sageattn_noalloc_status(stream_ptr(cuda)) == QF2_ERR_TIMEOUT
        assert lib.qf2_sageattn_noalloc_status(stream_ptr(cuda)) == 0
    finally:
        lib.qf2_sage_fault_injection(0, -1)
    got = _noalloc(lib, q, k, v, sm)
    assert lib.qf2_sageattn_noalloc_status(stream_ptr(cuda)) == 0
    assert torch.equal(got, _with_workspace(lib, q, k, v, sm))
