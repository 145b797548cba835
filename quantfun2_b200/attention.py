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
           "blocksparse_attn", "flash_attn", "do_attn", "unpad_tokens", "pad_tokens", "ATTN"]


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


# ------------------------------------------------ the attention processor seam --
# Backend of do_attn, as the reference's module global ATTN (src/models/common/attn.py:15):
# "b200" / "sage" -> Sage INT8/FP8 attention, "flash" / "sdpa" -> bf16 tcgen05 attention.
ATTN = "b200"


def flash_attn(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, softmax_scale: float | None = None,
               tensor_layout: str = "NHD") -> torch.Tensor:
    """Dense bf16 / fp16 attention on the tensor cores (tcgen05 kind::f16, exact online
    softmax, fp32 accumulation): the block-sparse kernel with every key block kept.  The
    counterpart of the reference's flash / SDPA branches (src/models/common/attn.py:92-107,
    123-130) for unmasked batches.  D = 128; equal query and key lengths."""
    B, Hq, S, D, _ = _hnd(q, tensor_layout)
    nb = (S + BLOCK - 1) // BLOCK
    idx = torch.arange(nb, dtype=torch.int32, device=q.device).expand(B, Hq, nb, nb).contiguous()
    return blocksparse_attn(q, k, v, idx, sm_scale=softmax_scale, tensor_layout=tensor_layout)


def unpad_tokens(x: torch.Tensor, mask: torch.Tensor):
    """x [B, S, H, D], key-padding mask [B, S] (True = token) -> (packed [B*S, H, D] whose
    first sum(mask) rows are the tokens in order, cu_seqlens int32 [B+1], dest int64 [B, S]:
    each token's packed row, B*S for padding).  All on the device, no host sync (the
    reference's _upad_input, src/misc/padding.py:75-182, reads the lengths back with .item())."""
    B, S = mask.shape
    m = mask.to(torch.bool)
    counts = m.sum(1, dtype=torch.int32)
    cu = torch.zeros(B + 1, dtype=torch.int32, device=x.device)
    cu[1:] = torch.cumsum(counts, 0, dtype=torch.int32)
    pos = torch.cumsum(m, 1, dtype=torch.int64) - 1
    dest = torch.where(m, cu[:-1, None].to(torch.int64) + pos, torch.full_like(pos, B * S))
    packed = torch.empty(B * S + 1, *x.shape[2:], dtype=x.dtype, device=x.device)
    packed.index_copy_(0, dest.reshape(-1), x.reshape(B * S, *x.shape[2:]))
    return packed[:B * S], cu, dest


def pad_tokens(packed_out: torch.Tensor, dest: torch.Tensor) -> torch.Tensor:
    """Inverse of unpad_tokens: [B*S, H, D] packed rows -> [B, S, H, D], zeros at padding
    (as the reference's pad_input)."""
    B, S = dest.shape
    full = torch.cat([packed_out, packed_out.new_zeros(1, *packed_out.shape[1:])], 0)
    return full.index_select(0, dest.reshape(-1)).view(B, S, *packed_out.shape[1:])


def do_attn(attn, xq: torch.Tensor, xk: torch.Tensor, xv: torch.Tensor, attn_mask: torch.Tensor | None,
            apply_fn=None, batch: int | None = None, seq_len: int | None = None,
            softmax_scale: float | None = None) -> torch.Tensor:
    """Mirror of the reference's _do_attn (src/models/common/attn.py:59-130) for the B200
    kernels: xq [B, S, Hq, D], xk / xv [B, S, Hkv, D] (NHD), attn_mask [B, S] key padding
    (True = token, None = all tokens) -> [B, S, Hq, D].  ATTN "b200" / "sage": Sage INT8/FP8
    attention, through the varlen kernel on the unpadded tokens when the mask pads (no
    host sync, padded rows of the output are zero); "flash" / "sdpa": bf16 attention on the
    tensor cores (unpadded batches).  `attn`, `apply_fn`, `batch` and `seq_len` are
    accepted for signature parity (the reference builds the SDPA mask with apply_fn)."""
    D = xq.shape[-1]
    if softmax_scale is None:
        softmax_scale = 1.0 / math.sqrt(D)
    if ATTN in ("flash", "sdpa"):
        if attn_mask is not None:
            raise QF2Error("the bf16 attention path takes unpadded batches; use ATTN='b200' for padded ones")
        return flash_attn(xq, xk, xv, softmax_scale, tensor_layout="NHD")
    if ATTN not in ("b200", "sage"):
        raise QF2Error(f"unknown ATTN backend {ATTN!r}")
    if attn_mask is None:
        return sageattn(xq, xk, xv, tensor_layout="NHD", sm_scale=softmax_scale)
    B, S = attn_mask.shape
    pq, cu, dest = unpad_tokens(xq, attn_mask)
    pk, _, _ = unpad_tokens(xk, attn_mask)
    pv, _, _ = unpad_tokens(xv, attn_mask)
    o = sageattn_varlen(pq, pk, pv, cu, cu, S, S, sm_scale=softmax_scale)
    return pad_tokens(o, dest)
