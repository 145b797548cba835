"""ctypes binding of libqf2b200.so (the C ABI declared in include/qf2b200.h).

The library is built in-tree by ``quantfun2_b200/build.py``.  There is no CPU or
PyTorch fallback: if the shared object is missing, or the current device is not
an sm_100 part, every op raises.
"""
from __future__ import annotations

import ctypes
import os
from ctypes import c_float, c_int, c_int64, c_void_p, POINTER
from pathlib import Path

# QF2_LIBRARY may name another build of the same library (same C ABI), e.g. one compiled
# with different tuning macros; the default is the in-tree build.
LIB_PATH = Path(os.environ.get("QF2_LIBRARY") or Path(__file__).resolve().parent / "libqf2b200.so")

QF2_OK = 0
QF2_F32, QF2_F16, QF2_BF16, QF2_I8, QF2_E4M3, QF2_I32 = range(6)
QF2_ROPE_FP16_TRIG = 1
QF2_RMS_EAGER, QF2_RMS_FUSED = 0, 1

_P64 = POINTER(c_int64)
_P32 = POINTER(ctypes.c_int32)

# name -> (restype, argtypes); mirrors include/qf2b200.h
SIGNATURES = {
    "qf2_version": (ctypes.c_char_p, []),
    "qf2_status_string": (ctypes.c_char_p, [c_int]),
    "qf2_last_error": (ctypes.c_char_p, []),
    "qf2_device_check": (c_int, []),
    "qf2_workspace_status": (c_int, [c_void_p, c_void_p]),
    "qf2_rope_apply": (
        c_int,
        [c_void_p, c_void_p, c_int64, _P64, _P64, c_void_p, c_void_p, c_int64, _P64, _P64, c_void_p, _P64,
         c_int64, c_int64, c_int64, c_int, c_int, c_void_p],
    ),
    "qf2_rms_gate_residual": (
        c_int,
        [c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64, c_void_p, c_float, c_void_p, c_int64, c_int,
         c_void_p, c_float, c_void_p, c_int64, c_void_p],
    ),
    "qf2_qkv_norm_rope": (
        c_int,
        [c_void_p, c_int64, c_int64, c_int64, c_int64, c_int64, c_int64, c_int64, c_void_p, _P64, c_void_p, _P64,
         c_void_p, _P64, c_void_p, c_void_p, c_float, c_void_p, _P64, c_void_p],
    ),
    "qf2_rmsnorm": (
        c_int,
        [c_void_p, c_int64, c_int, c_void_p, c_int, c_void_p, c_int64, c_int, c_int64, c_int64, c_float, c_int,
         c_void_p],
    ),
    "qf2_softmax_inplace": (c_int, [c_void_p, c_int64, c_int64, c_int64, c_int, c_void_p]),
    "qf2_sage_workspace_bytes": (
        c_int64, [c_int64, c_int64, c_int64, c_int64, c_int64, c_int64, c_int64, c_int64]),
    "qf2_sage_workspace_layout": (
        c_int, [c_int64, c_int64, c_int64, c_int64, c_int64, c_int64, c_int64, c_int64, _P64]),
    "qf2_sageattn": (
        c_int,
        [c_void_p, _P64, c_void_p, _P64, c_void_p, _P64, c_void_p, _P64, c_int64, c_int64, c_int64, c_int64,
         c_int64, c_int64, c_float, c_int, c_void_p, c_int64, c_void_p],
    ),
    "qf2_sageattn_varlen": (
        c_int,
        [c_void_p, _P64, c_void_p, _P64, c_void_p, _P64, c_void_p, _P64, _P32, _P32, c_int64, c_int64, c_int64,
         c_int64, c_int64, c_int64, c_int64, c_int64, c_float, c_int, c_void_p, c_int64, c_void_p],
    ),
    "qf2_sage_quantize": (
        c_int,
        [c_void_p, _P64, c_void_p, _P64, c_void_p, _P64, _P32, _P32, c_int64, c_int64, c_int64, c_int64, c_int64,
         c_int64, c_int64, c_int64, c_int64, c_int64, c_float, c_int, c_void_p, c_int64, c_void_p],
    ),
    "qf2_sage_attn_quantized": (
        c_int,
        [c_void_p, _P64, _P32, _P32, c_int64, c_int64, c_int64, c_int64, c_int64, c_int64, c_int64, c_int64,
         c_int64, c_int64, c_int, c_void_p, c_int64, c_void_p],
    ),
    "qf2_blocktopk_workspace_bytes": (c_int64, [c_int64, c_int64, c_int64, c_int64, c_int64]),
    "qf2_blocktopk_select": (
        c_int,
        [c_void_p, _P64, c_void_p, _P64, c_int64, c_int64, c_int64, c_int64, c_int64, c_int64, c_int, c_void_p,
         c_void_p, c_int64, c_void_p],
    ),
    "qf2_blocksparse_attn": (
        c_int,
        [c_void_p, _P64, c_void_p, _P64, c_void_p, _P64, c_void_p, _P64, c_int64, c_int64, c_int64, c_int64,
         c_int64, c_void_p, c_int64, c_float, c_int, c_void_p, c_int64, c_void_p],
    ),
    "qf2_quantize_rows": (
        c_int, [c_void_p, c_int64, c_int, c_int64, c_int64, c_void_p, c_int64, c_int, c_void_p, c_void_p]),
    "qf2_codes_to_bf16": (c_int, [c_void_p, c_int64, c_int, c_int64, c_int64, c_void_p, c_int64, c_void_p]),
    "qf2_gemm": (
        c_int,
        [c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_int64, c_int64, c_int64, c_int64, c_int, c_int,
         c_void_p, c_void_p, c_void_p, c_int, c_void_p, c_int64, c_void_p],
    ),
    "qf2_quantize_weight_rows": (
        c_int, [c_void_p, c_int64, c_int, c_int64, c_int64, c_void_p, c_int64, c_int, c_void_p, c_void_p]),
    "qf2_codes_convert": (
        c_int, [c_void_p, c_int64, c_int, c_int64, c_int64, c_void_p, c_int64, c_int, c_void_p]),
    "qf2_gemm_rows_indexed": (
        c_int,
        [c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_int64, c_int64, c_int64, c_int64, c_int64, c_int, c_int,
         c_void_p, c_int64, c_void_p, c_void_p, c_int, c_void_p, c_int64, c_void_p]),
    "qf2_rope_scatter": (
        c_int,
        [c_void_p, _P64, c_void_p, c_int64, c_void_p, c_void_p, _P64, c_int64, c_int64, c_int64, c_int64, c_int64,
         c_int, c_void_p, c_void_p]),
    "qf2_gemm_codes": (
        c_int,
        [c_void_p, c_int64, c_void_p, c_int64, c_int, c_void_p, c_int64, c_int64, c_int64, c_int64, c_int, c_int,
         c_void_p, c_void_p, c_void_p, c_int, c_int64, c_int, c_void_p, c_int64, c_void_p, c_int64, c_int64,
         c_void_p, c_int64, c_void_p],
    ),
    "qf2_gemm_ex": (
        c_int,
        [c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_int64, c_int64, c_int64, c_int64, c_int, c_int,
         c_void_p, c_void_p, c_void_p, c_int, c_int64, c_int, c_void_p, c_int64, c_void_p, c_int64, c_int64,
         c_void_p, c_int64, c_void_p],
    ),
    "qf2_ln_modulate": (
        c_int,
        [c_void_p, c_int64, c_int, c_void_p, c_void_p, c_int64, c_int64, c_int64, c_int64, c_float, c_void_p,
         c_int64, c_int, c_void_p, c_void_p],
    ),
    "qf2_copy_chunks": (c_int, [c_void_p, c_void_p, c_int64, _P64, _P64, _P64, c_void_p]),
    "qf2_sageattn_noalloc": (
        c_int,
        [c_void_p, _P64, c_void_p, _P64, c_void_p, _P64, c_void_p, _P64, c_int64, c_int64, c_int64, c_int64,
         c_int64, c_int64, c_float, c_int, c_void_p],
    ),
    "qf2_sageattn_noalloc_status": (c_int, [c_void_p]),
    "qf2_sage_fault_injection": (c_int, [c_int64, c_int]),
}

_lib = None


class QF2Error(RuntimeError):
    pass


def load() -> ctypes.CDLL:
    """Load the shared library (once) and bind every declared entry point."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise QF2Error(
            f"{LIB_PATH} is missing; build it with `python quantfun2_b200/build.py` "
            "(there is no CPU fallback)")
    lib = ctypes.CDLL(str(LIB_PATH))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def check(status: int, what: str) -> None:
    if status != QF2_OK:
        lib = load()
        msg = lib.qf2_status_string(status).decode()
        if status == -3:
            msg += ": " + lib.qf2_last_error().decode()
        raise QF2Error(f"{what} failed: {msg} ({status})")


def i64(*vals) -> ctypes.Array:
    return (c_int64 * len(vals))(*[int(v) for v in vals])


def ptr32(t) -> ctypes._Pointer:
    return ctypes.cast(c_void_p(t.data_ptr()), _P32)


_device_ok: dict[int, bool] = {}


def require_device(t) -> None:
    """Raise unless `t` lives on an sm_100 CUDA device."""
    import torch

    if not t.is_cuda:
        raise QF2Error("quantfun2_b200 ops run on CUDA tensors only (no CPU fallback)")
    idx = t.device.index if t.device.index is not None else torch.cuda.current_device()
    ok = _device_ok.get(idx)
    if ok is None:
        ok = torch.cuda.get_device_capability(idx) == (10, 0)
        _device_ok[idx] = ok
    if not ok:
        raise QF2Error(f"device {idx} is not compute capability 10.0 (B200); sm_100a kernels only")


def stream_ptr(device=None) -> c_void_p:
    import torch

    return c_void_p(torch.cuda.current_stream(device).cuda_stream)


def dtype_code(dt) -> int:
    import torch

    m = {torch.float32: QF2_F32, torch.float16: QF2_F16, torch.bfloat16: QF2_BF16}
    if dt not in m:
        raise QF2Error(f"unsupported dtype {dt}")
    return m[dt]


def header_symbols(header: str | os.PathLike | None = None) -> list[str]:
    """Function names declared in include/qf2b200.h."""
    import re

    h = Path(header) if header else Path(__file__).resolve().parent.parent / "include" / "qf2b200.h"
    text = h.read_text()
    return sorted(set(re.findall(r"^\s*(?:const\s+)?[a-z0-9_]+\*?\s+\*?(qf2_[a-z0-9_]+)\s*\(", text, re.M)))
