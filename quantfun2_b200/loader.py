"""Quantize-on-load: checkpoint tensors straight into the device-side quantized layouts.

Mirror of Pipelinelike.create_quantized_model_from_safetensors (src/pipeline.py:289-340):
the model arrives on the meta device, is cast to the qdtype's activation dtype, and is
materialised module by module; every nn.Linear selected by the filter is converted by the
qdtype (here: its weight becomes a QuantizedWeight of int8 / e4m3 codes and fp32 row
scales), every other parameter is loaded as it is.  Same arguments, same tensor naming
(module path + parameter name, rewritten by `replace_map`), same error on a missing
tensor (ValueError).

B200 side: each tensor is read from the memory-mapped file into a pinned staging buffer
by a host thread while the previous one is uploaded and quantized, uploaded once with an
asynchronous copy on a side stream, and quantized on the device by
qf2_quantize_weight_rows (torchao 0.7.0's steps in the activation dtype, the same codes
quantize_model produces from a loaded model); the float weight is dropped right after.
Device memory at peak: the quantized model plus one float weight.

The reference's GGUF path (src/pipeline.py:217-287) is not mirrored: as written it calls
the tuples of its _CONV_MAP (:24-34) as converters and feeds raw quantized GGUF blocks to
module_load, so it runs for no quantized GGUF file.
"""
from __future__ import annotations

from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

import torch
from torch import nn

from ._lib import QF2Error
from .quant import _nil, qdtype

__all__ = ["create_quantized_model_from_safetensors"]


def _walk(model: nn.Module, filt, cur_fqn: str = ""):
    """Modules in the reference's order (src/pipeline.py:315-336): a module's own
    parameters, then -- unless the filter selects it -- its children."""
    yield model, cur_fqn, bool(filt(model, cur_fqn[:-1]))
    if filt(model, cur_fqn[:-1]):
        return
    for name, child in model.named_children():
        yield from _walk(child, filt, f"{cur_fqn}{name}.")


@torch.no_grad()
def create_quantized_model_from_safetensors(meta_model: nn.Module, safetensors_file, device="cuda",
                                            quantization_device="cuda", dtype: qdtype | None = None,
                                            replace_map: dict[str, str] | None = None, skip=_nil) -> nn.Module:
    """Build `meta_model` (parameters on the meta device) from a safetensors checkpoint,
    quantizing its linears with `dtype` (a qdtype: qint8, qfloat8, qfloat8_w8a8)."""
    from safetensors import safe_open

    if dtype is None:
        raise QF2Error("a qdtype is required")
    replace_map = replace_map or {}
    convert, torch_dtype = dtype()
    meta_model.to(dtype=torch_dtype)
    device = torch.device(device)
    copy_stream = torch.cuda.Stream(device) if device.type == "cuda" else None

    def name_of(fqn: str, k: str) -> str:
        n = f"{fqn}{k}"
        for old, new in replace_map.items():
            n = n.replace(old, new)
        return n

    plan = list(_walk(meta_model, skip))
    with safe_open(str(Path(safetensors_file)), framework="pt", device="cpu") as f:
        keys = set(f.keys())
        names = [(mod, fqn, sel, k, name_of(fqn, k)) for mod, fqn, sel in plan
                 for k, _ in mod.named_parameters(recurse=False)]
        for *_, tname in names:
            if tname not in keys:
                raise ValueError(f"failed to load {tname}")

        def stage(tname: str) -> torch.Tensor:
            t = f.get_tensor(tname)
            host = torch.empty(t.shape, dtype=t.dtype, pin_memory=copy_stream is not None)
            host.copy_(t)
            return host

        with ThreadPoolExecutor(max_workers=1) as pool:
            pending = pool.submit(stage, names[0][4]) if names else None
            i = 0
            for mod, fqn, sel in plan:
                mod.to_empty(device=device, recurse=False)
                for k, param in mod.named_parameters(recurse=False):
                    host = pending.result()
                    i += 1
                    pending = pool.submit(stage, names[i][4]) if i < len(names) else None
                    if copy_stream is not None:
                        copy_stream.wait_stream(torch.cuda.current_stream(device))
                        with torch.cuda.stream(copy_stream):
                            dev = host.to(device, non_blocking=True)
                        torch.cuda.current_stream(device).wait_stream(copy_stream)
                        dev.record_stream(torch.cuda.current_stream(device))
                    else:
                        dev = host
                    param.copy_(dev.to(dtype=torch_dtype if param.is_floating_point() else param.dtype))
                if sel:
                    parent, _, child = fqn[:-1].rpartition(".")
                    new = convert(mod, device=device, quant_device=quantization_device)
                    if new is not mod:
                        owner = meta_model.get_submodule(parent) if parent else meta_model
                        setattr(owner, child, new)
    return meta_model
