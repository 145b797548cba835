"""Drop-in kernel ops for the reference's kernel seam (src/kernels/__init__.py).

The reference binds each op once, at import, through
``implemented_as(cuda_func=..., triton_func=...)`` (src/kernels/module.py:42-54).
This module exposes the same op names, argument meaning and return convention,
backed by libqf2b200.so (sm_100a CUDA).  There is no CPU or Triton fallback: the
ops raise ``QF2Error`` when the library is missing or the tensor is not on a
B200.

  rope_apply(xq, xk, freqs_cis)        -> (xq_out, xk_out)   __init__.py:126-142
  rope_apply_(xq, xk, freqs_cis)       -> (xq, xk) in place   triton/rope.py:83-134
  rmsnorm_apply(x, weight, eps)        -> Tensor              __init__.py:73-80
  inplace_softmax(x, dim=-1)           -> x                   __init__.py:83-87
  topk_attn(xq, xk, xv, mask, ...)     -> (out, POS_DICT)     __init__.py:146-195 (block form)
"""
from __future__ import annotations

import math

import torch

from . import _lib
from ._lib import QF2Error, check, dtype_code, i64, require_device, stream_ptr

__all__ = [
    "copy_chunks",
    "implemented_as",
    "rope_apply",
    "rope_apply_",
    "rmsnorm_apply",
    "inplace_softmax",
    "topk_attn",
    "qkv_norm_rope",
    "rms_gate_residual",
    "QF2Error",
]


def implemented_as(cuda_func=None, triton_func=None):
    """Same contract as the reference decorator (src/kernels/module.py:42-54): the
    decorated eager body is replaced at decoration time.  Here the sm_100a body
    (`cuda_func`) always wins; `triton_func` is accepted for signature parity and
    ignored (no Triton on this path)."""

    def decorator(func):
        impl = cuda_func if cuda_func is not None else func

        def inner(*args, **kwargs):
            return impl(*args, **kwargs)

        inner.__name__ = getattr(func, "__name__", "op")
        inner.__doc__ = getattr(impl, "__doc__", None)
        return inner

    return decorator


def _freqs_view(freqs_cis: torch.Tensor, B: int, S: int, half: int):
    if not freqs_cis.is_complex():
        freqs_cis = torch.view_as_complex(freqs_cis.contiguous())
    if freqs_cis.dtype != torch.complex64:
        freqs_cis = freqs_cis.to(torch.complex64)
    if freqs_cis.dim() == 2:
        freqs_cis = freqs_cis.unsqueeze(0)
    if freqs_cis.dim() != 3 or freqs_cis.shape[-1] != half or freqs_cis.shape[1] != S:
        raise QF2Error(f"freqs_cis shape {tuple(freqs_cis.shape)} does not match [B, {S}, {half}]")
    if freqs_cis.stride(-1) != 1:
        freqs_cis = freqs_cis.contiguous()
    fb = freqs_cis.shape[0]
    if fb not in (1, B):
        raise QF2Error(f"freqs_cis batch {fb} does not broadcast to {B}")
    sb = 0 if fb == 1 else freqs_cis.stride(0)
    return freqs_cis, (sb, freqs_cis.stride(1))


def _rope(xq, xk, freqs_cis, out_q, out_k, fp16_trig: bool):
    require_device(xq)
    if xq.dim() != 4 or (xk is not None and xk.dim() != 4):
        raise QF2Error("rope_apply expects [B, S, H, D] tensors")
    B, S, Hq, D = xq.shape
    if xq.stride(-1) != 1 or out_q.stride(-1) != 1:
        raise QF2Error("rope_apply needs a contiguous last dim")
    fc, fs = _freqs_view(freqs_cis.to(xq.device), B, S, D // 2)
    has_k = xk is not None
    if has_k:
        if xk.shape[0] != B or xk.shape[1] != S or xk.shape[3] != D or xk.dtype != xq.dtype:
            raise QF2Error("xk must match xq in batch, seq, head_dim and dtype")
        if xk.stride(-1) != 1 or out_k.stride(-1) != 1:
            raise QF2Error("rope_apply needs a contiguous last dim")
    Hk = xk.shape[2] if has_k else 0
    st = check(
        _lib.load().qf2_rope_apply(
            xq.data_ptr(), out_q.data_ptr(), Hq, i64(*xq.stride()[:3]), i64(*out_q.stride()[:3]),
            xk.data_ptr() if has_k else None, out_k.data_ptr() if has_k else None, Hk,
            i64(*xk.stride()[:3]) if has_k else None, i64(*out_k.stride()[:3]) if has_k else None,
            fc.data_ptr(), i64(*fs), B, S, D, dtype_code(xq.dtype),
            _lib.QF2_ROPE_FP16_TRIG if fp16_trig else 0, stream_ptr(xq.device)),
        "qf2_rope_apply")
    return st


def rope_apply(xq: torch.Tensor, xk: torch.Tensor, freqs_cis: torch.Tensor):
    """Eager-body semantics (src/kernels/__init__.py:126-142): returns new tensors,
    inputs untouched; fp32 rotation rounded to the input dtype."""
    out_q = torch.empty_like(xq)
    out_k = torch.empty_like(xk) if xk is not None else None
    _rope(xq, xk, freqs_cis, out_q, out_k, fp16_trig=False)
    return out_q, out_k


def rope_apply_(xq: torch.Tensor, xk: torch.Tensor, freqs_cis: torch.Tensor, fp16_trig: bool = True):
    """Triton-body semantics (src/kernels/triton/rope.py:83-134): rotates in place and
    returns the same tensors; cos/sin rounded to fp16 as rope_triton does."""
    _rope(xq, xk, freqs_cis, xq, xk, fp16_trig=fp16_trig)
    return xq, xk


def rmsnorm_apply(x: torch.Tensor, weight: torch.Tensor, eps: float, fused: bool = False) -> torch.Tensor:
    """x * rsqrt(mean(x^2, -1) + eps) * weight over the last dim.

    Default: the eager body's rounding (src/kernels/__init__.py:74-80): the
    normalized row is rounded to x.dtype, multiplied by weight, and the result has
    the promoted dtype of (x, weight).  fused=True: the Triton body's rounding
    (src/kernels/triton/rmsnorm.py:62-68): one rounding to x.dtype at the end.
    """
    require_device(x)
    N = weight.shape[0]
    if x.shape[-1] != N:
        raise QF2Error(f"last dim {x.shape[-1]} != weight size {N}")
    x2 = x.reshape(-1, N)
    if x2.stride(-1) != 1:
        x2 = x2.contiguous()
    w = weight.to(x.device)
    if w.stride(0) != 1:
        w = w.contiguous()
    out_dtype = x.dtype if fused else torch.promote_types(x.dtype, w.dtype)
    out = torch.empty(x.shape, dtype=out_dtype, device=x.device)
    o2 = out.view(-1, N)
    check(
        _lib.load().qf2_rmsnorm(
            x2.data_ptr(), x2.stride(0), dtype_code(x.dtype), w.data_ptr(), dtype_code(w.dtype), o2.data_ptr(),
            o2.stride(0), dtype_code(out_dtype), x2.shape[0], N, float(eps),
            _lib.QF2_RMS_FUSED if fused else _lib.QF2_RMS_EAGER, stream_ptr(x.device)),
        "qf2_rmsnorm")
    return out


def inplace_softmax(x: torch.Tensor, dim: int = -1) -> torch.Tensor:
    """Row softmax over the last dim, written back into x (src/kernels/__init__.py:83-87).
    Like the Triton wrapper (src/kernels/triton/softmax.py:82-91), a non-contiguous
    input is first made contiguous and the contiguous copy is returned."""
    if dim not in (-1, x.dim() - 1):
        raise QF2Error("Only dim=-1 is supported")
    require_device(x)
    if not x.is_contiguous():
        x = x.contiguous()
    n = x.shape[-1]
    rows = x.numel() // max(n, 1)
    check(_lib.load().qf2_softmax_inplace(x.data_ptr(), rows, n, n, dtype_code(x.dtype), stream_ptr(x.device)),
          "qf2_softmax_inplace")
    return x


def topk_attn(xq, xk, xv, mask, fn, HEAD_DIM, scale=None, TOP_K=256, POS_DICT=None, N_HEADS=32, N_KV_HEADS=8):
    """Block-sparse replacement of the reference's topk_attn (src/kernels/__init__.py:146-195).

    Same call and return convention: xq [B, S, Hq, D], xk/xv [B, S, Hkv, D] ->
    (out [B, S, Hq, D], POS_DICT).  Selection is per 128-token block: every query block
    keeps ceil(TOP_K / 128) key blocks ranked by mean-pooled Q . K^T; POS_DICT is the
    int32 block-index tensor [B, Hq, ceil(S/128), keep], computed when None and reused
    otherwise (the reference's layer-to-layer cache).  The inputs are not modified (the
    reference transposes them in place).  Key padding masks are not supported: `mask`
    must be None or all True.
    """
    from .attention import block_topk_select, blocksparse_attn

    if mask is not None and not bool(mask.all()):
        raise QF2Error("block-sparse topk_attn supports unpadded sequences only")
    if scale is None:
        scale = 1.0 / math.sqrt(HEAD_DIM)
    if POS_DICT is None:
        keep = max(1, -(-int(TOP_K) // 128))
        POS_DICT = block_topk_select(xq, xk, keep, tensor_layout="NHD")
    out = blocksparse_attn(xq, xk, xv, POS_DICT, sm_scale=scale, tensor_layout="NHD")
    return out, POS_DICT


def qkv_norm_rope(qkv: torch.Tensor, H: int, q_weight: torch.Tensor, k_weight: torch.Tensor,
                  freqs_cis: torch.Tensor, q_out: torch.Tensor, k_out: torch.Tensor, v_out: torch.Tensor,
                  eps: float = 1e-6, Hkv: int | None = None) -> None:
    """Fused per-head RMSNorm of q and k, RoPE of q and k, copy of v.
    qkv [B, L, (H + 2*Hkv)*head_dim] bf16 (q heads, then k heads, then v heads) ->
    q_out [B, L, H, Dout], k_out / v_out [B, L, Hkv, Dout] views (any strides with 16-byte
    rows, e.g. slices of a joint txt+img buffer); Dout >= head_dim is zero-padded."""
    require_device(qkv)
    Hkv = H if Hkv is None else Hkv
    B, L, W = qkv.shape
    head_dim = W // (H + 2 * Hkv)
    Dout = q_out.shape[-1]
    q2 = qkv.reshape(B * L, -1)
    if q2.stride(-1) != 1:
        q2 = q2.contiguous()
    fc, fs = _freqs_view(freqs_cis.to(qkv.device), B, L, head_dim // 2)
    st = lambda t: i64(t.stride(0), t.stride(1), t.stride(2))  # noqa: E731
    check(_lib.load().qf2_qkv_norm_rope(
        q2.data_ptr(), q2.stride(0), B, L, H, Hkv, head_dim, Dout, q_out.data_ptr(), st(q_out), k_out.data_ptr(),
        st(k_out), v_out.data_ptr(), st(v_out), q_weight.contiguous().data_ptr(), k_weight.contiguous().data_ptr(),
        float(eps), fc.data_ptr(), i64(*fs), stream_ptr(qkv.device)), "qf2_qkv_norm_rope")


def rms_gate_residual(x: torch.Tensor, y: torch.Tensor | None = None, h: torch.Tensor | None = None,
                      rows_per_batch: int | None = None, w_post: torch.Tensor | None = None, eps_post: float = 1e-5,
                      gate: torch.Tensor | None = None, gate_tanh: bool = True, w_pre: torch.Tensor | None = None,
                      eps_pre: float = 1e-5, scale: torch.Tensor | None = None) -> torch.Tensor | None:
    """The Lumina joint block's glue (src/models/lumina/image_two/model.py:82-101) in one pass
    over contiguous bf16 rows x [M, dim] (dim % 256 == 0):
        x += g * RMSNorm(y; w_post)      (in place; g = tanh(gate[b]) / gate[b] / 1)
        h  = RMSNorm(x; w_pre) * (1 + scale[b])
    gate / scale: [M / rows_per_batch, dim] bf16 views (row-strided).  Returns h."""
    require_device(x)
    M, dim = x.shape
    rpb = M if rows_per_batch is None else rows_per_batch
    for t in (x, y, h):
        if t is not None and (not t.is_contiguous() or t.dtype != torch.bfloat16 or t.shape != (M, dim)):
            raise QF2Error("x, y, h must be contiguous bf16 [M, dim]")
    for t in (gate, scale):
        if t is not None and (t.stride(-1) != 1 or t.dtype != torch.bfloat16):
            raise QF2Error("gate / scale must be bf16 row-strided views")
    p = lambda t: None if t is None else t.data_ptr()  # noqa: E731
    wp = None if w_post is None else w_post.to(torch.bfloat16).contiguous()
    wq = None if w_pre is None else w_pre.to(torch.bfloat16).contiguous()
    check(_lib.load().qf2_rms_gate_residual(
        p(y), x.data_ptr(), p(h), M, dim, rpb, p(wp), float(eps_post or 0.0), p(gate),
        0 if gate is None else gate.stride(0), int(bool(gate_tanh)), p(wq), float(eps_pre or 0.0), p(scale),
        0 if scale is None else scale.stride(0), stream_ptr(x.device)), "qf2_rms_gate_residual")
    return h


def copy_chunks(dst: torch.Tensor, src: torch.Tensor, chunk_bytes: int, dims, src_strides, dst_strides) -> None:
    """Chunk permutation copy on the device: dims (up to 4, last fastest) index the chunks
    of chunk_bytes bytes; chunk i goes from src's byte offset sum(i_k * src_strides[k]) to
    dst's sum(i_k * dst_strides[k]).  Byte strides; everything 16-byte aligned."""
    require_device(dst)
    d, ss, ds = list(dims), list(src_strides), list(dst_strides)
    while len(d) < 4:
        d.insert(0, 1)
        ss.insert(0, 0)
        ds.insert(0, 0)
    check(_lib.load().qf2_copy_chunks(dst.data_ptr(), src.data_ptr(), int(chunk_bytes), i64(*d), i64(*ss), i64(*ds),
                                      stream_ptr(dst.device)), "qf2_copy_chunks")


def rope_scatter(x: torch.Tensor, f: torch.Tensor, idx: torch.Tensor, y: torch.Tensor) -> torch.Tensor:
    """RoPE of the reference's RAS partial ops (PYCUDA_ROPE_KERNEL, src/kernels/cuda/ras.cu:
    12-52): y[b, idx[n], h] = x[b, n, h] rotated by f[n] for x [B, N, H, D] bf16, f [N, D]
    fp32 (interleaved cos, sin per pair; a leading 1 dim is accepted), idx int64 [N] and the
    destination y [B, M, H, D] bf16, updated in place (rows not in idx untouched).
    Raises QF2Error when an index lies outside [0, M) (that row is skipped)."""
    require_device(x)
    B, N, H, D = x.shape
    M = y.shape[1]
    f2 = f.reshape(-1, f.shape[-1]).to(device=x.device, dtype=torch.float32)
    if f2.stride(-1) != 1:
        f2 = f2.contiguous()
    if f2.shape != (N, D):
        raise QF2Error(f"f must be [N, D] = [{N}, {D}] floats")
    ix = idx.to(device=x.device, dtype=torch.int64).contiguous()
    ws = torch.zeros(64, dtype=torch.int32, device=x.device)
    st = lambda t: i64(t.stride(0), t.stride(1), t.stride(2))  # noqa: E731
    lib = _lib.load()
    check(lib.qf2_rope_scatter(x.data_ptr(), st(x), f2.data_ptr(), f2.stride(0), ix.data_ptr(), y.data_ptr(), st(y),
                               B, N, M, H, D, _lib.dtype_code(x.dtype), ws.data_ptr(), stream_ptr(x.device)),
          "qf2_rope_scatter")
    check(lib.qf2_workspace_status(ws.data_ptr(), stream_ptr(x.device)), "qf2_rope_scatter (index range)")
    return y


def partially_linear(x: torch.Tensor, w: torch.Tensor, index: torch.Tensor, out: torch.Tensor | None = None,
                     check_index: bool = True) -> torch.Tensor:
    """Row-indexed linear of the reference's RAS partial ops (_partially_linear,
    src/kernels/triton/ras.py:100-128): out[b, index[m]] = x[b, m] . w^T for x [B, M, K],
    w [N, K] (bf16 or fp16, same dtype), index int64 [M].  `out` [B, M_out, N] is updated in
    place (rows not in index untouched); without it a new [B, M, N] tensor is returned
    whose unindexed rows are uninitialized (the reference returns torch.empty_like(x)).
    check_index=True synchronizes to report an index outside [0, M_out)."""
    require_device(x)
    B, M, K = x.shape
    N = w.shape[0]
    if w.shape[1] != K or w.dtype != x.dtype:
        raise QF2Error("w must be [N, K] in x's dtype")
    if out is None:
        out = torch.empty(B, M, N, dtype=x.dtype, device=x.device)
    if out.dim() != 3 or out.shape[0] != B or out.shape[2] != N or out.stride(2) != 1 or \
            out.stride(0) != out.shape[1] * out.stride(1):
        raise QF2Error("out must be [B, M_out, N] with contiguous rows and batches")
    x2 = x.reshape(B * M, K)
    if x2.stride(-1) != 1 or x2.stride(0) != K:
        x2 = x2.contiguous()
    wc = w.contiguous()
    ix = index.to(device=x.device, dtype=torch.int64).contiguous()
    ws = torch.zeros(64, dtype=torch.int32, device=x.device)
    lib = _lib.load()
    check(lib.qf2_gemm_rows_indexed(x2.data_ptr(), K, wc.data_ptr(), K, out.data_ptr(), out.stride(1), B, M, N, K,
                                    _lib.dtype_code(x.dtype), _lib.dtype_code(out.dtype), ix.data_ptr(), out.shape[1],
                                    None, None, _lib.QF2_F32, ws.data_ptr(), 256, stream_ptr(x.device)),
          "qf2_gemm_rows_indexed")
    if check_index:
        check(lib.qf2_workspace_status(ws.data_ptr(), stream_ptr(x.device)), "qf2_gemm_rows_indexed (index range)")
    return out
