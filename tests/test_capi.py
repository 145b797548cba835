"""CPU: the C-ABI library loads, exports every symbol include/qf2b200.h declares, and
rejects bad arguments before touching the device."""
import ctypes

import pytest

from quantfun2_b200 import _lib


def test_library_exports_every_header_symbol():
    lib = _lib.load()
    syms = _lib.header_symbols()
    assert len(syms) >= 10
    for s in syms:
        assert hasattr(lib, s), s
    assert set(syms) == set(_lib.SIGNATURES), "ctypes signature table out of sync with the header"


def test_version_and_status_strings():
    lib = _lib.load()
    assert b"sm_100a" in lib.qf2_version()
    assert lib.qf2_status_string(-4) == b"a bounded device-side wait timed out"
    assert lib.qf2_status_string(12345) == b"unknown status"


def test_argument_validation_without_device():
    lib = _lib.load()
    s = _lib.i64(0, 0, 0)
    assert lib.qf2_rmsnorm(None, 0, 0, None, 0, None, 0, 0, 1, 1, 1e-6, 0, None) == -8
    assert lib.qf2_rmsnorm(ctypes.c_void_p(16), 0, 0, ctypes.c_void_p(16), 0, ctypes.c_void_p(16), 0, 0, 1, 0,
                           1e-6, 0, None) == -1
    assert lib.qf2_softmax_inplace(None, 1, 1, 1, 0, None) == -8
    assert lib.qf2_rope_apply(None, None, 1, s, s, None, None, 0, None, None, None, s, 1, 1, 2, 0, 0, None) == -8
    assert lib.qf2_sage_workspace_bytes(1, 24, 24, 4608, 4608, 4608, 4608, 80) == -1   # D in {64, 96, 128}
    assert lib.qf2_sage_workspace_bytes(1, 24, 24, 4608, 4608, 4608, 4608, 96) > 0
    p = ctypes.c_void_p(1024)
    # an unsupported D and a bad dtype are rejected before any launch
    assert lib.qf2_sageattn(p, s, p, s, p, s, p, s, 1, 2, 2, 64, 64, 48, 0.1, 2, p, 1 << 30, None) == -1
    assert lib.qf2_sageattn(p, s, p, s, p, s, p, s, 1, 2, 2, 64, 64, 128, 0.1, 0, p, 1 << 30, None) == -2
    assert lib.qf2_sageattn(p, s, p, s, p, s, p, s, 1, 3, 2, 64, 64, 128, 0.1, 2, p, 1 << 30, None) == -1  # GQA ratio
    assert lib.qf2_sageattn(p, s, p, s, p, s, p, s, 1, 2, 2, 64, 64, 128, 0.1, 2, p, 16, None) == -6        # workspace


def test_sage_workspace_layout_is_consistent():
    lib = _lib.load()
    offs = _lib.i64(*([0] * 12))
    B, H, S = 2, 24, 4608
    assert lib.qf2_sage_workspace_layout(B, H, H, -1, -1, S, S, 128, offs) == 0
    o = list(offs)
    assert o == sorted(o) and all(x % 1024 == 0 for x in o)
    tiles = B * ((S + 127) // 128)
    assert o[2] - o[1] == H * tiles * 16384          # q codes
    assert lib.qf2_sage_workspace_bytes(B, H, H, B * S, B * S, S, S, 128) >= o[11]


def test_device_check_reports_missing_device():
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    assert _lib.load().qf2_device_check() == -7


def test_loader_reports_a_missing_tensor(tmp_path):
    """create_quantized_model_from_safetensors names the tensor it cannot find, before
    anything is allocated or quantized (src/pipeline.py:325-327 raises ValueError too)."""
    import torch
    from safetensors.torch import save_file

    from quantfun2_b200.loader import create_quantized_model_from_safetensors
    from quantfun2_b200.quant import qint8

    lin = torch.nn.Sequential(torch.nn.Linear(8, 16), torch.nn.Linear(16, 8))
    sd = {k: v for k, v in lin.state_dict().items() if k != "1.bias"}
    save_file(sd, str(tmp_path / "m.safetensors"))
    with torch.device("meta"):
        meta = torch.nn.Sequential(torch.nn.Linear(8, 16), torch.nn.Linear(16, 8))
    with pytest.raises(ValueError, match="1.bias"):
        create_quantized_model_from_safetensors(meta, tmp_path / "m.safetensors", device="cpu", dtype=qint8)
