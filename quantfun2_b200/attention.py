"""Attention ops behind the reference's attention-processor seam.

The reference picks its attention backend with the module global ``ATTN``
(src/models/common/attn.py:15, read again by src/models/flux/attn.py:6) and, for
``ATTN == "sage"``, calls the third-party sageattention package:

  sageattn(q, k, v)                                   src/models/flux/attn.py:39-41
  sageattn_varlen(q, k, v, cu_seqlens_q, cu_seqlens_k,
                  max_seqlen_q, max_seqlen_k, sm_scale) src/models/common/attn.py:109-120

This module provides both with the package's argument meaning (layouts "HND" /
"NHD", packed varlen [T, H, D], GQA by head ratio), backed by the sm_100a kernels
in libqf2b200.so.  The workspace (quantized codes and scales) is allocated by
PyTorch's caching allocator for each call; the library itself allocates nothing.
"""
from __future__ import annotations

import math

import torch

from . import _lib
from ._lib import QF2Error, check, i64, ptr32, require_device, stream_ptr

__all__ = ["sageattn", "sageattn_varlen", "sage_quantize", "sage_workspace_layout", "block_topk_select",
           "blocksparse_attn"]


def _dt(t: torch.Tensor) -> int:
    if t.dtype == torch.bfloat16:
        return _lib.QF2_BF16
    if t.dtype == torch.float16:
        return _lib.QF2_F16
    raise QF2Error(f"sageattn supports bf16/fp16 inputs, got {t.dtype}")


def _fix(t: torch.Tensor) -> torch.Tensor:
    # 16-byte rows: last dim contiguous and every stride a multiple of 8 elements
    if t.stride(-1) != 1 or any(s % 8 for s in t.stride()[:-1]) or t.data_ptr() % 16:
        t = t.contiguous()
    return t


def _workspace(nbytes: int, device) -> torch.Tensor:
    # 1024-byte aligned start (the caching allocator returns 512-byte aligned blocks)
    raw = torch.empty(nbytes + 1024, dtype=torch.uint8, device=device)
    off = (-raw.data_ptr()) % 1024
    return raw[off:off + nbytes]


def sageattn(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, tensor_layout: str = "HND",
             is_causal: bool = False, sm_scale: float | None = None, return_lse: bool = False,
             out: torch.Tensor | None = None, **kwargs) -> torch.Tensor:
    """INT8 QK^T / FP8 PV attention.  q [B, Hq, Sq, D] (HND) or [B, Sq, Hq, D] (NHD);
    k, v with Hkv heads (Hq % Hkv == 0).  D = 64, 96 or 128.  Returns a tensor in q's layout;
    `out` may be any strided view of that shape (16-byte aligned rows)."""
    if is_causal:
        raise QF2Error("causal masking is not on the DiT path (bidirectional attention only)")
    if return_lse:
        raise QF2Error("return_lse is not supported")
    require_device(q)
    q, k, v = _fix(q), _fix(k), _fix(v)
    if tensor_layout == "HND":
        B, Hq, Sq, D = q.shape
        Hkv, Skv = k.shape[1], k.shape[2]
        perm = lambda t: (t.stride(0), t.stride(1), t.stride(2))  # noqa: E731
    elif tensor_layout == "NHD":
        B, Sq, Hq, D = q.shape
        Skv, Hkv = k.shape[1], k.shape[2]
        perm = lambda t: (t.stride(0), t.stride(2), t.stride(1))  # noqa: E731
    else:
        raise QF2Error(f"unknown tensor_layout {tensor_layout}")
    if v.shape != k.shape or k.dtype != q.dtype or v.dtype != q.dtype:
        raise QF2Error("k and v must have the same shape, and q/k/v the same dtype")
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(D)
    if out is None:
        out = torch.empty_like(q)
    elif out.shape != q.shape or out.dtype != q.dtype or out.stride(-1) != 1:
        raise QF2Error("out must match q's shape and dtype with a contiguous last dim")
    lib = _lib.load()
    nbytes = lib.qf2_sage_workspace_bytes(B, Hq, Hkv, B * Sq, B * Skv, Sq, Skv, D)
    if nbytes < 0:
        check(int(nbytes), "qf2_sage_workspace_bytes")
    ws = _workspace(int(nbytes), q.device)
    check(
        lib.qf2_sageattn(q.data_ptr(), i64(*perm(q)), k.data_ptr(), i64(*perm(k)), v.data_ptr(), i64(*perm(v)),
                         out.data_ptr(), i64(*perm(out)), B, Hq, Hkv, Sq, Skv, D, float(sm_scale), _dt(q),
                         ws.data_ptr(), ws.numel(), stream_ptr(q.device)),
        "qf2_sageattn")
    return out


def sageattn_varlen(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, cu_seqlens_q: torch.Tensor,
                    cu_seqlens_k: torch.Tensor, max_seqlen_q: int, max_seqlen_k: int, is_causal: bool = False,
                    sm_scale: float | None = None, smooth_k: bool = True, **kwargs) -> torch.Tensor:
    """Packed variable-length form: q [Tq, Hq, D], k/v [Tk, Hkv, D], cu_seqlens int32 [batch+1]."""
    if is_causal:
        raise QF2Error("causal masking is not on the DiT path (bidirectional attention only)")
    if not smooth_k:
        raise QF2Error("K smoothing is always applied on this path")
    require_device(q)
    q, k, v = _fix(q), _fix(k), _fix(v)
    Tq, Hq, D = q.shape
    Tk, Hkv, _ = k.shape
    batch = cu_seqlens_q.numel() - 1
    cu_q = cu_seqlens_q.to(device=q.device, dtype=torch.int32).contiguous()
    cu_k = cu_seqlens_k.to(device=q.device, dtype=torch.int32).contiguous()
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(D)
    out = torch.empty_like(q)
    lib = _lib.load()
    nbytes = lib.qf2_sage_workspace_bytes(batch, Hq, Hkv, Tq, Tk, int(max_seqlen_q), int(max_seqlen_k), D)
    if nbytes < 0:
        check(int(nbytes), "qf2_sage_workspace_bytes")
    ws = _workspace(int(nbytes), q.device)
    st2 = lambda t: (t.stride(0), t.stride(1))  # noqa: E731
    check(
        lib.qf2_sageattn_varlen(q.data_ptr(), i64(*st2(q)), k.data_ptr(), i64(*st2(k)), v.data_ptr(), i64(*st2(v)),
                                out.data_ptr(), i64(*st2(out)), ptr32(cu_q), ptr32(cu_k), batch, Tq, Tk,
                                int(max_seqlen_q), int(max_seqlen_k), Hq, Hkv, D, float(sm_scale), _dt(q),
                                ws.data_ptr(), ws.numel(), stream_ptr(q.device)),
        "qf2_sageattn_varlen")
    return out


def sage_workspace_layout(batch, Hq, Hkv, Sq, Skv, D=128, varlen_totals=None):
    """Byte offsets of the workspace regions (status, q codes, q scales, k codes, k scales,
    v codes, v scales, k mean, v inverse scales, split-KV partial rows, split-KV row max/sum, total)."""
    offs = i64(*([0] * 12))
    if varlen_totals is None:
        check(_lib.load().qf2_sage_workspace_layout(batch, Hq, Hkv, -1, -1, Sq, Skv, D, offs), "layout")
    else:
        tq, tk = varlen_totals
        check(_lib.load().qf2_sage_workspace_layout(batch, Hq, Hkv, tq, tk, Sq, Skv, D, offs), "layout")
    return [int(x) for x in offs]


def sage_quantize(q, k, v, sm_scale=None, tensor_layout="HND", cu_seqlens_q=None, cu_seqlens_k=None,
                  max_seqlen_q=None, max_seqlen_k=None):
    """Run only the quantization stage; returns (workspace uint8 tensor, layout offsets)."""
    require_device(q)
    q, k, v = _fix(q), _fix(k), _fix(v)
    lib = _lib.load()
    if cu_seqlens_q is None:
        if tensor_layout == "HND":
            B, Hq, Sq, D = q.shape
            Hkv, Skv = k.shape[1], k.shape[2]
            perm = lambda t: (t.stride(0), t.stride(1), t.stride(2))  # noqa: E731
        else:
            B, Sq, Hq, D = q.shape
            Skv, Hkv = k.shape[1], k.shape[2]
            perm = lambda t: (t.stride(0), t.stride(2), t.stride(1))  # noqa: E731
        sm_scale = 1.0 / math.sqrt(D) if sm_scale is None else sm_scale
        nbytes = lib.qf2_sage_workspace_bytes(B, Hq, Hkv, B * Sq, B * Skv, Sq, Skv, D)
        ws = _workspace(int(nbytes), q.device)
        check(lib.qf2_sage_quantize(q.data_ptr(), i64(*perm(q)), k.data_ptr(), i64(*perm(k)), v.data_ptr(),
                                    i64(*perm(v)), None, None, B, Sq, Skv, 0, 0, 0, 0, Hq, Hkv, D, float(sm_scale),
                                    _dt(q), ws.data_ptr(), ws.numel(), stream_ptr(q.device)), "qf2_sage_quantize")
        return ws, sage_workspace_layout(B, Hq, Hkv, Sq, Skv, D)
    Tq, Hq, D = q.shape
    Tk, Hkv, _ = k.shape
    batch = cu_seqlens_q.numel() - 1
    cu_q = cu_seqlens_q.to(device=q.device, dtype=torch.int32).contiguous()
    cu_k = cu_seqlens_k.to(device=q.device, dtype=torch.int32).contiguous()
    sm_scale = 1.0 / math.sqrt(D) if sm_scale is None else sm_scale
    nbytes = lib.qf2_sage_workspace_bytes(batch, Hq, Hkv, Tq, Tk, int(max_seqlen_q), int(max_seqlen_k), D)
    ws = _workspace(int(nbytes), q.device)
    st2 = lambda t: (t.stride(0), t.stride(1), 0)  # noqa: E731
    check(lib.qf2_sage_quantize(q.data_ptr(), i64(*st2(q)), k.data_ptr(), i64(*st2(k)), v.data_ptr(), i64(*st2(v)),
                                ptr32(cu_q), ptr32(cu_k), batch, 0, 0, Tq, Tk, int(max_seqlen_q), int(max_seqlen_k),
                                Hq, Hkv, D, float(sm_scale), _dt(q), ws.data_ptr(), ws.numel(),
                                stream_ptr(q.device)), "qf2_sage_quantize")
    return ws, sage_workspace_layout(batch, Hq, Hkv, int(max_seqlen_q), int(max_seqlen_k), D, (Tq, Tk))


# ------------------------------------------------------ top-k block sparse --
BLOCK = 128


def _hnd(t: torch.Tensor, layout: str):
    """(B, H, S, D) view and {batch, head, seq} strides of a q/k/v tensor."""
    if layout == "HND":
        return t.shape[0], t.shape[1], t.shape[2], t.shape[3], (t.stride(0), t.stride(1), t.stride(2))
    if layout == "NHD":
        return t.shape[0], t.shape[2], t.shape[1], t.shape[3], (t.stride(0), t.stride(2), t.stride(1))
    raise QF2Error(f"unknown tensor_layout {layout}")


def block_topk_select(q: torch.Tensor, k: torch.Tensor, keep: int, tensor_layout: str = "HND") -> torch.Tensor:
    """Kept key blocks per 128-token query block: int32 [B, Hq, ceil(S/128), keep], ascending.
    Block scores are mean-pooled Q . mean-pooled K^T (fp64, rounded to fp32); the lower block
    index wins ties."""
    require_device(q)
    q, k = _fix(q), _fix(k)
    B, Hq, S, D, qs = _hnd(q, tensor_layout)
    _, Hkv, Sk, _, ks = _hnd(k, tensor_layout)
    if Sk != S:
        raise QF2Error("block top-k needs equal query and key lengths")
    nb = (S + BLOCK - 1) // BLOCK
    keep = min(int(keep), nb)
    idx = torch.empty(B, Hq, nb, keep, dtype=torch.int32, device=q.device)
    lib = _lib.load()
    nbytes = int(lib.qf2_blocktopk_workspace_bytes(B, Hq, Hkv, S, D))
    if nbytes < 0:
        check(nbytes, "qf2_blocktopk_workspace_bytes")
    ws = torch.empty(nbytes, dtype=torch.uint8, device=q.device)
    check(lib.qf2_blocktopk_select(q.data_ptr(), i64(*qs), k.data_ptr(), i64(*ks), B, Hq, Hkv, S, D, keep, _dt(q),
                                   idx.data_ptr(), ws.data_ptr(), nbytes, stream_ptr(q.device)),
          "qf2_blocktopk_select")
    return idx


def blocksparse_attn(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, idx: torch.Tensor,
                     sm_scale: float | None = None, tensor_layout: str = "HND") -> torch.Tensor:
    """Exact softmax attention of each 128-row query block over its kept key blocks `idx`."""
    require_device(q)
    q, k, v = _fix(q), _fix(k), _fix(v)
    B, Hq, S, D, qs = _hnd(q, tensor_layout)
    _, Hkv, _, _, ks = _hnd(k, tensor_layout)
    _, _, _, _, vs = _hnd(v, tensor_layout)
    if v.shape != k.shape or k.dtype != q.dtype or v.dtype != q.dtype:
        raise QF2Error("k and v must have the same shape, and q/k/v the same dtype")
    nb = (S + BLOCK - 1) // BLOCK
    if idx.dim() != 4 or tuple(idx.shape[:3]) != (B, Hq, nb) or idx.dtype != torch.int32:
        raise QF2Error(f"idx must be int32 [B, Hq, {nb}, keep]")
    idx = idx.to(q.device).contiguous()
    out = torch.empty_like(q)
    _, _, _, _, os_ = _hnd(out, tensor_layout)
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(D)
    ws = torch.empty(256, dtype=torch.uint8, device=q.device)
    check(_lib.load().qf2_blocksparse_attn(q.data_ptr(), i64(*qs), k.data_ptr(), i64(*ks), v.data_ptr(), i64(*vs),
                                           out.data_ptr(), i64(*os_), B, Hq, Hkv, S, D, idx.data_ptr(),
                                           idx.shape[3], float(sm_scale), _dt(q), ws.data_ptr(), 256,
                                           stream_ptr(q.device)),
          "qf2_blocksparse_attn")
    return out
