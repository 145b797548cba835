"""Quantized linears behind the reference's quantization seam (src/quant.py).

The reference picks a `qdtype` (qint8 / qfloat8 ..., src/quant.py:318-360) and
`quantize_model` (:402-412) walks the model, swapping torchao weight subclasses into
every nn.Linear (linear_inserter, :131-148).  Here the same names build QLinear
modules whose forward runs the sm_100a kernels of libqf2b200.so:

  qint8      weight-only INT8: per-output-row symmetric codes; y = (x . bf16(codes)^T) * s_w + b
  qfloat8    weight-only FP8 e4m3: per-output-row codes; same GEMM on bf16 copies of the codes
  qfloat8_w8a8  FP8 e4m3 weights and per-token e4m3 activations on the FP8 tensor cores:
             y = (e4m3(x) . codes^T) * s_x * s_w + b

Activations are bf16 (the reference casts int8/float8 models to fp16, `supported_dtypes`
at :326,331; the B200 kernels run bf16).
"""
from __future__ import annotations

import types
from dataclasses import dataclass, field
from functools import partial

import torch
from torch import nn

from . import _lib
from ._lib import QF2Error, check, require_device, stream_ptr

__all__ = ["qdtype", "QLinear", "qint8", "qfloat8", "qfloat8_w8a8", "quantize_model", "linear_inserter",
           "quantize_rows", "codes_to_bf16", "gemm", "ln_modulate", "glu_interleave"]


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
         glu: bool = False) -> torch.Tensor:
    """D = (a . b^T) * row_scale[:, None] * col_scale[None, :] + bias on tcgen05.
    a [M, K], b [N, K]: bf16, or uint8 e4m3 codes with fp8=True.
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
    check(_lib.load().qf2_gemm_ex(
        a.data_ptr(), a.stride(0), b.data_ptr(), b.stride(0), out.data_ptr(), out.stride(0), M, N, K,
        _lib.QF2_E4M3 if fp8 else _lib.QF2_BF16, _lib.QF2_F32 if out_dtype == torch.float32 else _lib.QF2_BF16,
        row_scale.data_ptr() if row_scale is not None else None,
        col_scale.data_ptr() if col_scale is not None else None,
        bias.data_ptr() if bias is not None else None, bias_dt, int(gelu_col0), int(bool(glu)),
        residual.data_ptr() if residual is not None else None, residual.stride(0) if residual is not None else 0,
        gate.data_ptr() if gate is not None else None, gate.stride(0) if gate is not None else 0,
        int(rows_per_gate), ws.data_ptr(), 256, stream_ptr(a.device)),
        "qf2_gemm_ex")
    return out


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


class QLinear(nn.Module):
    """nn.Linear replacement holding per-output-row quantized weights.
    mode: "int8" (weight-only), "fp8" (weight-only e4m3), "fp8_w8a8" (e4m3 weights and activations)."""

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
        codes, scale = quantize_rows(w, "int8" if mode == "int8" else "e4m3")
        bias = None if lin.bias is None else lin.bias.detach().to(w.device, torch.bfloat16)
        return cls(codes, scale, bias, mode, lin.in_features, lin.out_features)

    @property
    def fp8_activations(self) -> bool:
        return self.mode == "fp8_w8a8"

    def prep(self, x2: torch.Tensor):
        """Activation operand for this linear: (e4m3 codes, per-row scales) or (bf16, None)."""
        if x2.dtype != torch.bfloat16:
            x2 = x2.to(torch.bfloat16)
        if self.fp8_activations:
            return quantize_rows(x2, "e4m3")
        return x2, None

    def prep_ln_modulate(self, x2, shift, scale, rows_per_batch):
        """Fused LayerNorm + modulate producing this linear's activation operand."""
        if self.fp8_activations:
            return ln_modulate(x2, shift, scale, rows_per_batch, "e4m3")
        return ln_modulate(x2, shift, scale, rows_per_batch, "bf16"), None

    def run(self, a: torch.Tensor, row_scale, **epilogue) -> torch.Tensor:
        """GEMM on a prepared operand; epilogue kwargs as in `gemm` (out, gelu_col0, residual, gate...)."""
        if self.fp8_activations:
            return gemm(a, self.codes, row_scale=row_scale, col_scale=self.scale, bias=self.bias, fp8=True, **epilogue)
        wb = codes_to_bf16(self.codes, "int8" if self.mode == "int8" else "e4m3")
        return gemm(a, wb, col_scale=self.scale, bias=self.bias, **epilogue)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        shape = x.shape
        y = self.run(*self.prep(x.reshape(-1, shape[-1])))
        return y.reshape(*shape[:-1], self.out_features)

    def extra_repr(self) -> str:
        return f"in_features={self.in_features}, out_features={self.out_features}, mode={self.mode}"


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


def linear_inserter(mode: str):
    """Mirror of src/quant.py:131-148: returns a function that converts one nn.Linear."""

    def insert(lin: nn.Linear, device=None, quant_device=None):
        return QLinear.from_linear(lin, mode, device=quant_device or device)

    return insert


qint8 = qdtype("int8", partial(linear_inserter, "int8"), supported_dtypes=[torch.bfloat16])
qfloat8 = qdtype("float8", partial(linear_inserter, "fp8"), supported_dtypes=[torch.bfloat16])
qfloat8_w8a8 = qdtype("float8_w8a8", partial(linear_inserter, "fp8_w8a8"), supported_dtypes=[torch.bfloat16])


def _nil(module: nn.Module, fqn: str) -> bool:
    return isinstance(module, nn.Linear)


def _replace(model: nn.Module, replacement_map, filter_fn, cur_fqn: str, device, quant_device):
    if filter_fn(model, cur_fqn[:-1]):
        conv, dt = (replacement_map[cur_fqn[:-1]] if isinstance(replacement_map, dict) else replacement_map)()
        return conv(model.to(dtype=dt), device=device, quant_device=quant_device)
    for name, child in model.named_children():
        new = _replace(child, replacement_map, filter_fn, f"{cur_fqn}{name}.", device, quant_device)
        if new is not child:
            setattr(model, name, new)
    return model


def quantize_model(model: nn.Module, dtype_map, device="cuda", quantization_device="cuda", skip=_nil) -> nn.Module:
    """Mirror of src/quant.py:402-412: every module selected by `skip` (default: every
    nn.Linear) is replaced by the converter of `dtype_map` (a qdtype, or a dict from
    module path to qdtype); the rest of the model is moved to the qdtype's activation dtype."""
    model = _replace(model, dtype_map, skip, "", device, quantization_device)
    dt = (dtype_map if not isinstance(dtype_map, dict) else next(iter(dtype_map.values()))).supported_dtypes[0]
    for m in model.modules():
        if not isinstance(m, QLinear):
            for p in m.parameters(recurse=False):
                p.data = p.data.to(device=device, dtype=dt) if p.is_floating_point() else p.data.to(device)
    return model.to(device)
