"""Quantized linears behind the reference's quantization seam (src/quant.py).

The reference picks a `qdtype` (qint8 / qfloat8 ..., src/quant.py:318-360) and
`quantize_model` (:402-412) walks the model, casts each nn.Linear to the qdtype's
activation dtype (fp16 for qint8 / qfloat8, :326,331,383) and swaps a torchao weight
subclass into its `weight` (linear_inserter, :131-148), so F.linear dispatches to the
quantized matmul.  The same names here do the same with `QuantizedWeight`, a tensor
subclass whose F.linear runs the sm_100a kernels of libqf2b200.so:

  qint8      weight-only INT8: per-output-row symmetric codes; y = (x . codes^T) * s_w + b
  qfloat8    weight-only FP8 e4m3: per-output-row codes; same GEMM
  qfloat8_w8a8  FP8 e4m3 weights and per-token e4m3 activations on the FP8 tensor cores:
             y = (e4m3(x) . codes^T) * s_x * s_w + b   (no counterpart in the reference)

Weights are quantized by torchao 0.7.0's steps in the weight's dtype
(`qf2_quantize_weight_rows`).  Activations stay in their own dtype (fp16 or bf16): the
codes are expanded exactly to that dtype and the GEMM runs fp16 x fp16 or bf16 x bf16
on the tensor cores with fp32 accumulation, the per-channel scale and the bias in its
epilogue, and one rounding to the activation dtype.

`QLinear` is the module form the DiT steps of this package build directly (it adds the
fused LayerNorm-modulate prologue and the GEMM epilogues).
"""
from __future__ import annotations

import types
from dataclasses import dataclass, field
from functools import partial

import torch
import torch.nn.functional as F
from torch import nn

from . import _lib
from ._lib import QF2Error, check, require_device, stream_ptr

__all__ = ["qdtype", "QLinear", "QuantizedWeight", "qint8", "qfloat8", "qfloat8_w8a8", "quantize_model",
           "linear_inserter", "quantize_rows", "quantize_weight", "codes_to_bf16", "codes_to", "gemm",
           "ln_modulate", "glu_interleave"]


def _ws(device) -> torch.Tensor:
    return torch.empty(256, dtype=torch.uint8, device=device)


def quantize_rows(x: torch.Tensor, fmt: str):
    """Per-row symmetric quantization: fmt "int8" -> (int8 codes, fp32 scales) with
    scale = max(amax/127.5, eps); fmt "e4m3" -> (uint8 e4m3 codes, scales) with scale = amax/448."""
    require_device(x)
    x2 = x.reshape(-1, x.shape[-1])
    if x2.stride(-1) != 1:
        x2 = x2.contiguous()
    M, K = x2.shape
    q = torch.empty(M, K, dtype=torch.int8 if fmt == "int8" else torch.uint8, device=x.device)
    scales = torch.empty(M, dtype=torch.float32, device=x.device)
    check(_lib.load().qf2_quantize_rows(x2.data_ptr(), x2.stride(0), _lib.dtype_code(x.dtype), M, K, q.data_ptr(), K,
                                        _lib.QF2_I8 if fmt == "int8" else _lib.QF2_E4M3, scales.data_ptr(),
                                        stream_ptr(x.device)), "qf2_quantize_rows")
    return q, scales


def quantize_weight(w: torch.Tensor, fmt: str):
    """Per-output-row quantization of a weight [N, K] by torchao 0.7.0's steps, every step
    rounded in w's dtype (fp16, bf16 or fp32): fmt "int8" -> (int8 codes, fp32 scales),
    "e4m3" -> (uint8 e4m3 codes, fp32 scales)."""
    require_device(w)
    if w.dim() != 2:
        raise QF2Error("quantize_weight expects a 2-D weight")
    if w.stride(-1) != 1:
        w = w.contiguous()
    M, K = w.shape
    q = torch.empty(M, K, dtype=torch.int8 if fmt == "int8" else torch.uint8, device=w.device)
    scales = torch.empty(M, dtype=torch.float32, device=w.device)
    check(_lib.load().qf2_quantize_weight_rows(w.data_ptr(), w.stride(0), _lib.dtype_code(w.dtype), M, K,
                                               q.data_ptr(), K, _lib.QF2_I8 if fmt == "int8" else _lib.QF2_E4M3,
                                               scales.data_ptr(), stream_ptr(w.device)), "qf2_quantize_weight_rows")
    return q, scales


def codes_to(q: torch.Tensor, fmt: str, dtype: torch.dtype) -> torch.Tensor:
    """int8 / e4m3 codes -> exact bf16 or fp16 values."""
    require_device(q)
    M, K = q.shape
    out = torch.empty(M, K, dtype=dtype, device=q.device)
    check(_lib.load().qf2_codes_convert(q.data_ptr(), q.stride(0), _lib.QF2_I8 if fmt == "int8" else _lib.QF2_E4M3,
                                        M, K, out.data_ptr(), K, _lib.dtype_code(dtype), stream_ptr(q.device)),
          "qf2_codes_convert")
    return out


def codes_to_bf16(q: torch.Tensor, fmt: str) -> torch.Tensor:
    require_device(q)
    M, K = q.shape
    out = torch.empty(M, K, dtype=torch.bfloat16, device=q.device)
    check(_lib.load().qf2_codes_to_bf16(q.data_ptr(), q.stride(0), _lib.QF2_I8 if fmt == "int8" else _lib.QF2_E4M3,
                                        M, K, out.data_ptr(), K, stream_ptr(q.device)), "qf2_codes_to_bf16")
    return out


def gemm(a: torch.Tensor, b: torch.Tensor, row_scale=None, col_scale=None, bias=None, fp8: bool = False,
         out_dtype=torch.bfloat16, out: torch.Tensor | None = None, gelu_col0: int = -1,
         residual: torch.Tensor | None = None, gate: torch.Tensor | None = None, rows_per_gate: int = 1,
         glu: bool = False, codes: str | None = None) -> torch.Tensor:
    """D = (a . b^T) * row_scale[:, None] * col_scale[None, :] + bias on tcgen05.
    a [M, K], b [N, K]: both bf16, both fp16, or uint8 e4m3 codes with fp8=True; with
    codes="int8" / "e4m3", b holds 8-bit weight codes (int8 / uint8 e4m3, K % 16 == 0) that
    the kernel turns into a's 16-bit type in shared memory (exact), for weight-only linears.
    out_dtype bf16, fp16 or fp32 (fused residual / SwiGLU: bf16).
    Fused epilogue: GELU (tanh) on columns >= gelu_col0; D = residual + gate * D when
    residual is given (gate [rows/rows_per_gate, N] bf16, may be a strided view); with
    glu=True b holds SwiGLU weights in `glu_interleave` order and D = silu(gate) * up
    [M, N/2].  `out` may be a row-strided 2-D view (for instance a column slice of a
    larger buffer)."""
    require_device(a)
    M, K = a.shape
    N = b.shape[0]
    if b.shape[1] != K:
        raise QF2Error("inner dimensions differ")
    if codes is not None:
        if codes not in ("int8", "e4m3") or fp8 or a.dtype not in (torch.bfloat16, torch.float16):
            raise QF2Error("weight codes need a bf16 or fp16 activation operand")
        if b.dtype != (torch.int8 if codes == "int8" else torch.uint8):
            raise QF2Error("int8 codes are torch.int8, e4m3 codes torch.uint8")
    elif not fp8 and (a.dtype not in (torch.bfloat16, torch.float16) or b.dtype != a.dtype):
        raise QF2Error("16-bit GEMM operands must both be bf16 or both fp16")
    if a.stride(-1) != 1:
        a = a.contiguous()
    if b.stride(-1) != 1:
        b = b.contiguous()
    No = N // 2 if glu else N
    if out is None:
        out = torch.empty(M, No, dtype=out_dtype, device=a.device)
    elif out.shape != (M, No) or out.stride(-1) != 1 or out.dtype != out_dtype:
        raise QF2Error("out must be an [M, N] row-strided view of the output dtype")
    if residual is not None and (residual.stride(-1) != 1 or residual.dtype != torch.bfloat16):
        raise QF2Error("residual must be a bf16 row-strided [M, N] view")
    if gate is not None and (gate.stride(-1) != 1 or gate.dtype != torch.bfloat16):
        raise QF2Error("gate must be a bf16 row-strided view")
    bias_dt = _lib.QF2_F32
    if bias is not None:
        bias = bias.contiguous()
        bias_dt = _lib.QF2_BF16 if bias.dtype == torch.bfloat16 else _lib.QF2_F32
        if bias.dtype not in (torch.bfloat16, torch.float32):
            bias = bias.float()
    ws = _ws(a.device)
    tail = (row_scale.data_ptr() if row_scale is not None else None,
            col_scale.data_ptr() if col_scale is not None else None,
            bias.data_ptr() if bias is not None else None, bias_dt, int(gelu_col0), int(bool(glu)),
            residual.data_ptr() if residual is not None else None, residual.stride(0) if residual is not None else 0,
            gate.data_ptr() if gate is not None else None, gate.stride(0) if gate is not None else 0,
            int(rows_per_gate), ws.data_ptr(), 256, stream_ptr(a.device))
    if codes is not None:
        check(_lib.load().qf2_gemm_codes(
            a.data_ptr(), a.stride(0), b.data_ptr(), b.stride(0), _lib.QF2_I8 if codes == "int8" else _lib.QF2_E4M3,
            out.data_ptr(), out.stride(0), M, N, K, _lib.dtype_code(a.dtype), _lib.dtype_code(out_dtype), *tail),
            "qf2_gemm_codes")
        return out
    check(_lib.load().qf2_gemm_ex(
        a.data_ptr(), a.stride(0), b.data_ptr(), b.stride(0), out.data_ptr(), out.stride(0), M, N, K,
        _lib.QF2_E4M3 if fp8 else _lib.dtype_code(a.dtype), _lib.dtype_code(out_dtype), *tail),
        "qf2_gemm_ex")
    return out


def _weight_only(a: torch.Tensor, codes: torch.Tensor, fmt: str, scale, bias, **epilogue) -> torch.Tensor:
    """Weight-only linear on 8-bit codes: y = (a . fmt(codes)^T) * scale + bias in a's dtype.
    Up to 128 rows the codes go straight into the GEMM (converted in shared memory, one
    128-row tile of a); above that one expansion to a's dtype and the 16-bit GEMM are
    faster, since the in-GEMM conversion would repeat for every 128-row tile."""
    if a.shape[0] <= 128:
        return gemm(a, codes, col_scale=scale, bias=bias, out_dtype=a.dtype, codes=fmt, **epilogue)
    w = codes_to_bf16(codes, fmt) if a.dtype == torch.bfloat16 else codes_to(codes, fmt, a.dtype)
    return gemm(a, w, col_scale=scale, bias=bias, out_dtype=a.dtype, **epilogue)


def glu_interleave(w1: torch.Tensor, w3: torch.Tensor) -> torch.Tensor:
    """Rows of the SwiGLU gate (w1) and up (w3) projections [hidden, in] stacked in the
    order the glu epilogue reads them: for each 128-row block j, w1[128j:128j+128] then
    w3[128j:128j+128].  hidden % 128 == 0.  Works on codes, scales and biases alike."""
    if w1.shape != w3.shape or w1.shape[0] % 128:
        raise QF2Error("w1 / w3 must have equal shapes with hidden % 128 == 0")
    h = w1.shape[0]
    tail = w1.shape[1:]
    return torch.stack([w1.reshape(h // 128, 128, *tail), w3.reshape(h // 128, 128, *tail)], 1).reshape(2 * h, *tail)


def ln_modulate(x: torch.Tensor, shift: torch.Tensor, scale: torch.Tensor, rows_per_batch: int, fmt: str = "bf16",
                eps: float = 1e-6):
    """LayerNorm(x) * (1 + scale) + shift over the last dim of x [M, N] (shift/scale
    [M / rows_per_batch, N] bf16 views).  fmt "bf16" -> bf16 [M, N]; "e4m3" -> (uint8 codes,
    fp32 per-row scales) ready for the FP8 GEMM."""
    require_device(x)
    M, N = x.shape
    fp8 = fmt == "e4m3"
    out = torch.empty(M, N, dtype=torch.uint8 if fp8 else torch.bfloat16, device=x.device)
    scales = torch.empty(M, dtype=torch.float32, device=x.device) if fp8 else None
    if shift.stride(-1) != 1 or scale.stride(-1) != 1 or shift.stride(0) != scale.stride(0):
        raise QF2Error("shift and scale must be row-strided views with a common stride")
    check(_lib.load().qf2_ln_modulate(
        x.data_ptr(), x.stride(0), _lib.dtype_code(x.dtype), shift.data_ptr(), scale.data_ptr(), shift.stride(0),
        int(rows_per_batch), M, N, float(eps), out.data_ptr(), N, _lib.QF2_E4M3 if fp8 else _lib.QF2_BF16,
        scales.data_ptr() if fp8 else None, stream_ptr(x.device)), "qf2_ln_modulate")
    return (out, scales) if fp8 else out


def _check_act(x: torch.Tensor) -> None:
    if x.dtype not in (torch.float16, torch.bfloat16):
        raise QF2Error(f"quantized linears take fp16 or bf16 activations, got {x.dtype} "
                       "(the reference casts the model to the qdtype's dtype first)")


class QLinear(nn.Module):
    """nn.Linear replacement holding per-output-row quantized weights (the module form the
    DiT steps use).  mode: "int8" (weight-only), "fp8" (weight-only e4m3), "fp8_w8a8"
    (e4m3 weights and activations).  Activations run in their own dtype (fp16 or bf16)."""

    def __init__(self, codes: torch.Tensor, scale: torch.Tensor, bias: torch.Tensor | None, mode: str,
                 in_features: int, out_features: int):
        super().__init__()
        self.mode = mode
        self.in_features = in_features
        self.out_features = out_features
        self.register_buffer("codes", codes)
        self.register_buffer("scale", scale)
        self.register_buffer("bias", bias)

    @classmethod
    def from_linear(cls, lin: nn.Linear, mode: str, device=None) -> "QLinear":
        w = lin.weight.detach().to(device or lin.weight.device)
        if not w.is_cuda:
            raise QF2Error("quantize on a CUDA device (no CPU quantizer on this path)")
        codes, scale = quantize_weight(w, "int8" if mode == "int8" else "e4m3")
        bias = None if lin.bias is None else lin.bias.detach().to(w.device, torch.float32)
        return cls(codes, scale, bias, mode, lin.in_features, lin.out_features)

    @property
    def fp8_activations(self) -> bool:
        return self.mode == "fp8_w8a8"

    def prep(self, x2: torch.Tensor):
        """Activation operand for this linear: (e4m3 codes, per-row scales) or (x, None)."""
        _check_act(x2)
        if self.fp8_activations:
            return quantize_rows(x2, "e4m3")
        return x2, None

    def prep_ln_modulate(self, x2, shift, scale, rows_per_batch):
        """Fused LayerNorm + modulate producing this linear's activation operand (bf16)."""
        if self.fp8_activations:
            return ln_modulate(x2, shift, scale, rows_per_batch, "e4m3")
        return ln_modulate(x2, shift, scale, rows_per_batch, "bf16"), None

    def run(self, a: torch.Tensor, row_scale, out_dtype=torch.bfloat16, **epilogue) -> torch.Tensor:
        """GEMM on a prepared operand; epilogue kwargs as in `gemm` (out, gelu_col0, residual, gate...).
        A 16-bit operand sets the output dtype (its own); e4m3 operands use out_dtype."""
        if self.fp8_activations:
            return gemm(a, self.codes, row_scale=row_scale, col_scale=self.scale, bias=self.bias, fp8=True,
                        out_dtype=out_dtype, **epilogue)
        return _weight_only(a, self.codes, "int8" if self.mode == "int8" else "e4m3", self.scale, self.bias,
                            **epilogue)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        shape = x.shape
        y = self.run(*self.prep(x.reshape(-1, shape[-1])), out_dtype=x.dtype)
        return y.reshape(*shape[:-1], self.out_features)

    def extra_repr(self) -> str:
        return f"in_features={self.in_features}, out_features={self.out_features}, mode={self.mode}"


class QuantizedWeight(torch.Tensor):
    """Quantized nn.Linear weight, the counterpart of the torchao AffineQuantizedTensor the
    reference sets as `lin.weight` (src/quant.py:131-148).  It keeps the per-output-row
    codes and fp32 scales on the device and reports the weight's logical shape [out, in]
    and the activation dtype; F.linear(x, w, b) with this weight runs the tcgen05 GEMM
    (x in fp16 or bf16; mode "fp8_w8a8" quantizes x per token to e4m3 first).  Other ops
    are refused: there is no dequantize-to-float fallback.  `.to(device)` moves the codes;
    `.to(dtype)` changes the activation dtype (fp16 / bf16) without requantizing."""

    @staticmethod
    def __new__(cls, codes: torch.Tensor, scale: torch.Tensor, mode: str, dtype: torch.dtype, shape):
        return torch.Tensor._make_wrapper_subclass(cls, tuple(shape), dtype=dtype, device=codes.device,
                                                   requires_grad=False)

    def __init__(self, codes: torch.Tensor, scale: torch.Tensor, mode: str, dtype: torch.dtype, shape):
        self.codes = codes
        self.scale = scale
        self.mode = mode

    @classmethod
    def from_float(cls, w: torch.Tensor, mode: str) -> "QuantizedWeight":
        """Quantize a float weight [out, in] (on an sm_100 device) in its own dtype."""
        codes, scale = quantize_weight(w.detach(), "int8" if mode == "int8" else "e4m3")
        act = w.dtype if w.dtype in (torch.float16, torch.bfloat16) else torch.float16
        return cls(codes, scale, mode, act, w.shape)

    def __repr__(self, *, tensor_contents=None) -> str:  # noqa: D105
        return (f"QuantizedWeight(shape={tuple(self.shape)}, mode={self.mode}, act_dtype={self.dtype}, "
                f"device={self.device})")

    def _with(self, codes=None, scale=None, dtype=None) -> "QuantizedWeight":
        return QuantizedWeight(self.codes if codes is None else codes, self.scale if scale is None else scale,
                               self.mode, dtype or self.dtype, self.shape)

    def linear(self, x: torch.Tensor, bias: torch.Tensor | None = None) -> torch.Tensor:
        _check_act(x)
        require_device(x)
        N, K = self.shape
        x2 = x.reshape(-1, K)
        b = None if bias is None else bias.detach().float()
        if self.mode == "fp8_w8a8":
            xc, xs = quantize_rows(x2, "e4m3")
            y = gemm(xc, self.codes, row_scale=xs, col_scale=self.scale, bias=b, fp8=True, out_dtype=x.dtype)
        else:
            y = _weight_only(x2.contiguous() if x2.stride(-1) != 1 else x2, self.codes,
                             "int8" if self.mode == "int8" else "e4m3", self.scale, b)
        return y.reshape(*x.shape[:-1], N)

    @classmethod
    def __torch_function__(cls, func, types, args=(), kwargs=None):
        kwargs = kwargs or {}
        if func is F.linear:
            x, w = args[0], args[1]
            b = args[2] if len(args) > 2 else kwargs.get("bias")
            if not isinstance(w, QuantizedWeight) or isinstance(x, QuantizedWeight):
                raise QF2Error("F.linear with a QuantizedWeight expects it as the weight")
            return w.linear(x, b)
        if func is torch._has_compatible_shallow_copy_type:
            return False  # module.to() swaps the parameter instead of set_data (src/quant.py:85-90)
        with torch._C.DisableTorchFunctionSubclass():
            return func(*args, **kwargs)

    @classmethod
    def __torch_dispatch__(cls, func, types, args=(), kwargs=None):
        kwargs = kwargs or {}
        aten = torch.ops.aten
        w = args[0] if args else None
        if func is aten.detach.default or func is aten.alias.default:
            return w._with()
        if func is aten._to_copy.default:
            dev = kwargs.get("device") or w.device
            dt = kwargs.get("dtype") or w.dtype
            if dt not in (torch.float16, torch.bfloat16):
                raise QF2Error(f"a quantized weight runs fp16 or bf16 activations, not {dt}")
            return w._with(codes=w.codes.to(dev), scale=w.scale.to(dev), dtype=dt)
        if func is aten._has_compatible_shallow_copy_type.default:
            return False
        raise QF2Error(f"{func} is not defined on a quantized weight (only F.linear, detach and .to)")


@dataclass
class qdtype:
    """Same shape as the reference's qdtype (src/quant.py:93-128): calling it returns
    (linear converter, activation dtype)."""
    display: str
    apply_function: any
    args: list = field(default_factory=list)
    supported_dtypes: list = field(default_factory=list)

    def __repr__(self) -> str:
        return self.display

    def __call__(self, *args, layout: str = "default", **kwargs):
        self.args = args
        if layout != "default":
            raise QF2Error("only the default layout exists on this path")
        return self.apply_function(*args, **kwargs), self.supported_dtypes[0]


def linear_inserter(mode: str, allow_requires_grad: bool = False):
    """Mirror of src/quant.py:131-148: returns a function that quantizes one nn.Linear in
    place -- its weight becomes a QuantizedWeight parameter (on `device`, quantized on
    `quant_device`) and the module itself is kept, so state-dict keys do not change."""

    def insert(lin: nn.Linear, device=None, quant_device=None):
        device = device if device is not None else lin.weight.device
        quant_device = quant_device if quant_device is not None else lin.weight.device
        w = lin.weight.detach().to(device=quant_device)
        if not w.is_cuda:
            raise QF2Error("quantize on a CUDA device (no CPU quantizer on this path)")
        qw = QuantizedWeight.from_float(w, mode).to(device)
        lin.weight = nn.Parameter(qw, requires_grad=False)
        lin.extra_repr = types.MethodType(
            lambda self: f"in_features={self.in_features}, out_features={self.out_features}, "
                         f"weight={self.weight!r}", lin)
        return lin

    return insert


# activation dtypes as the reference's supported_dtypes (src/quant.py:323-332)
qint8 = qdtype("int8", partial(linear_inserter, "int8"), supported_dtypes=[torch.float16])
qfloat8 = qdtype("float8", partial(linear_inserter, "fp8"), supported_dtypes=[torch.float16])
qfloat8_w8a8 = qdtype("float8_w8a8", partial(linear_inserter, "fp8_w8a8"), supported_dtypes=[torch.bfloat16])


def _nil(module: nn.Module, fqn: str) -> bool:
    return isinstance(module, nn.Linear)


def _replace(model: nn.Module, replacement_map, filter_fn, cur_fqn: str, device, quant_device):
    """src/quant.py:368-399: the selected module is cast to the qdtype's activation dtype
    and converted; every other module is walked and then cast to that dtype."""
    if filter_fn(model, cur_fqn[:-1]):
        conv, dt = (replacement_map[cur_fqn] if isinstance(replacement_map, dict) else replacement_map)()
        return conv(model.to(dtype=dt), device=device, quant_device=quant_device).to(device=device)
    for name, child in model.named_children():
        new = _replace(child, replacement_map, filter_fn, f"{cur_fqn}{name}.", device, quant_device)
        if new is not child:
            setattr(model, name, new)
    if isinstance(replacement_map, dict):
        return model.to(replacement_map[cur_fqn]()[1])
    return model.to(replacement_map()[1])


def quantize_model(model: nn.Module, dtype_map, device="cuda", quantization_device="cuda", skip=_nil) -> nn.Module:
    """Mirror of src/quant.py:402-412: every module selected by `skip` (default: every
    nn.Linear) gets its weight quantized by the converter of `dtype_map` (a qdtype, or a
    dict from module path + "." to qdtype, as the reference indexes it); the model ends up
    in the qdtype's activation dtype."""
    _replace(model, dtype_map, skip, "", device, quantization_device)
    return model
