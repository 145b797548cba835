"""Generate golden vectors from the reference implementation itself.

Run in the build container, where the reference source tree is mounted:
    python tests/golden/make_golden.py <path of the quantfun2 source tree>
It imports the reference's eager kernel bodies (src/kernels/__init__.py) and its
JointAttention block (src/models/common/attn.py) on the CPU, using the import shim
the reference needs on a GPU-less host (triton absent -> eager bodies bound;
src.models package inits skipped because they import diffusers), runs them on
seeded inputs and writes tests/golden/ref_ops.npz and tests/golden/ref_jattn.npz.
bf16 tensors are stored as uint16 bit patterns.  The reference is not needed to *use*
the fixtures.
"""
from __future__ import annotations

import importlib
import math
import sys
import types
from pathlib import Path

import numpy as np
import torch

OUT = Path(__file__).resolve().parent / "ref_ops.npz"
OUT_JATTN = Path(__file__).resolve().parent / "ref_jattn.npz"

# JointAttention blocks at the attention kernel's head dims: (tag, dim, q heads, kv heads,
# seq, grid side).  Head dim 128 is the Flux / single-block configuration's, 96 Lumina's
# (24 q / 8 kv heads there, the same 3:1 grouping here).
JATTN_CASES = (("d128", 512, 4, 2, 320, 20), ("d96", 576, 6, 2, 320, 20))


def jattn_weights(dim: int, heads: int, kv_heads: int, seed: int) -> dict[str, torch.Tensor]:
    """Projection and norm weights of a JointAttention block, from a seeded CPU generator
    (uniform +-1/sqrt(in), the nn.Linear default range) and rounded to bf16 so a bf16
    device path holds them exactly.  The GPU test rebuilds them with this function."""
    g = torch.Generator().manual_seed(seed)
    hd = dim // heads
    shapes = {"wq": (heads * hd, dim), "wk": (kv_heads * hd, dim), "wv": (kv_heads * hd, dim),
              "wo": (dim, heads * hd)}
    w = {n: ((torch.rand(*sh, generator=g) * 2 - 1) / math.sqrt(sh[1])).bfloat16().float()
         for n, sh in shapes.items()}
    w["q_norm"] = (torch.rand(hd, generator=g) + 0.5).bfloat16().float()
    w["k_norm"] = (torch.rand(hd, generator=g) + 0.5).bfloat16().float()
    return w


def import_reference(root: str):
    import torch.utils._triton as tt

    tt.has_triton = lambda: True      # enter the try-branch of src/kernels/module.py:5-11 ...
    sys.modules["triton"] = None      # ... whose `import triton` then fails -> eager bodies
    sys.path.insert(0, root)
    importlib.import_module("src")
    for name in ["src.models", "src.models.common"]:
        m = types.ModuleType(name)
        m.__path__ = [str(Path(root) / name.replace(".", "/"))]
        sys.modules[name] = m
    kernels = importlib.import_module("src.kernels")
    attn = importlib.import_module("src.models.common.attn")
    lumina = importlib.import_module("src.models.lumina.image_two.model")
    attn.ATTN = "sdpa"
    return kernels, attn, lumina


def bf16_bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def main(root: str) -> None:
    K, A, L = import_reference(root)
    g = torch.Generator().manual_seed(1234)
    out: dict[str, np.ndarray] = {}

    # ---- RoPE: 3-axis freqs from the reference RopeEmbedder (model.py:105-151)
    B, S, Hq, Hk, D = 2, 37, 4, 2, 32
    emb = L.RopeEmbedder(theta=10000.0, axes_dims=(8, 12, 12), axes_lens=(64, 16, 16))
    ids = torch.zeros(B, S, 3, dtype=torch.int32)
    ids[:, :, 0] = torch.arange(S) % 64
    ids[:, :, 1] = (torch.arange(S) // 6) % 16
    ids[:, :, 2] = torch.arange(S) % 6
    ids[1] = ids[1].flip(0)
    freqs = emb(ids)                                   # complex64 [B, S, D/2]
    out["rope_freqs"] = torch.view_as_real(freqs).numpy()
    xq = torch.randn(B, S, Hq, D, generator=g)
    xk = torch.randn(B, S, Hk, D, generator=g)
    oq, ok = K.rope_apply(xq.clone(), xk.clone(), freqs)
    out["rope_f32_xq"], out["rope_f32_xk"] = xq.numpy(), xk.numpy()
    out["rope_f32_oq"], out["rope_f32_ok"] = oq.numpy(), ok.numpy()
    xqb, xkb = xq.bfloat16(), xk.bfloat16()
    oqb, okb = K.rope_apply(xqb.clone(), xkb.clone(), freqs)
    out["rope_bf16_xq"], out["rope_bf16_xk"] = bf16_bits(xqb), bf16_bits(xkb)
    out["rope_bf16_oq"], out["rope_bf16_ok"] = bf16_bits(oqb), bf16_bits(okb)

    # ---- RMSNorm (eager body, kernels/__init__.py:73-80)
    for tag, (shape, eps) in {"head": ((5, 7, 96), 1e-6), "row": ((3, 2304), 1e-5)}.items():
        x = torch.randn(*shape, generator=g) * 3.0
        w = torch.rand(shape[-1], generator=g) + 0.5
        out[f"rms_{tag}_x_f32"], out[f"rms_{tag}_w_f32"] = x.numpy(), w.numpy()
        out[f"rms_{tag}_y_f32"] = K.rmsnorm_apply(x, w, eps).numpy()
        xb, wb = x.bfloat16(), w.bfloat16()
        out[f"rms_{tag}_x_bf16"], out[f"rms_{tag}_w_bf16"] = bf16_bits(xb), bf16_bits(wb)
        out[f"rms_{tag}_y_bf16"] = bf16_bits(K.rmsnorm_apply(xb, wb, eps))
        out[f"rms_{tag}_eps"] = np.array([eps], dtype=np.float64)

    # ---- softmax (eager body, kernels/__init__.py:83-87)
    x = torch.randn(2, 3, 5, 300, generator=g) * 4.0
    out["softmax_x_f32"] = x.numpy()
    out["softmax_y_f32"] = K.inplace_softmax(x.clone(), -1).numpy()
    xb = x.bfloat16()
    out["softmax_x_bf16"] = bf16_bits(xb)
    out["softmax_y_bf16"] = bf16_bits(K.inplace_softmax(xb.clone(), -1))

    # ---- JointAttention block (common/attn.py:133-236), SDPA branch, fp32,
    #      a small version of the single-block CPU configuration
    torch.manual_seed(0)
    dim, heads, kv_heads, seq = 128, 2, 2, 48
    blk = A.JointAttention(0, 10000, dim, heads, kv_heads, qk_norm=True).eval()
    with torch.no_grad():
        blk.q_norm.weight.copy_(torch.rand(dim // heads, generator=g) + 0.5)
        blk.k_norm.weight.copy_(torch.rand(dim // heads, generator=g) + 0.5)
        x = torch.randn(1, seq, dim, generator=g)
        mask = torch.ones(1, seq, dtype=torch.bool)
        emb2 = L.RopeEmbedder(theta=10000.0, axes_dims=(16, 24, 24), axes_lens=(1, 8, 8))
        ids2 = torch.zeros(1, seq, 3, dtype=torch.int32)
        ids2[0, :, 1] = torch.arange(seq) // 8
        ids2[0, :, 2] = torch.arange(seq) % 8
        f2 = emb2(ids2)
        y = blk(x, mask, f2)
    out["jattn_x"] = x.numpy()
    out["jattn_freqs"] = torch.view_as_real(f2).numpy()
    for n in ["wq", "wk", "wv", "wo"]:
        out[f"jattn_{n}"] = getattr(blk, n).weight.detach().numpy()
    out["jattn_qnorm"] = blk.q_norm.weight.detach().numpy()
    out["jattn_knorm"] = blk.k_norm.weight.detach().numpy()
    out["jattn_y"] = y.numpy()
    out["jattn_meta"] = np.array([dim, heads, kv_heads, seq], dtype=np.int64)

    np.savez_compressed(OUT, **out)
    print(f"wrote {OUT} ({OUT.stat().st_size} bytes, {len(out)} arrays)")

    # ---- JointAttention at head dims 128 and 96 (common/attn.py:133-236), SDPA branch,
    #      fp32, GQA, 2-axis RoPE over a 16 x 20 grid (320 tokens: a ragged last 128-token tile);
    #      bf16-representable x and weights
    ja: dict[str, np.ndarray] = {}
    for i, (tag, dim, heads, kvh, seq, side) in enumerate(JATTN_CASES):
        hd = dim // heads
        blk = A.JointAttention(0, 10000, dim, heads, kvh, qk_norm=True).eval()
        w = jattn_weights(dim, heads, kvh, seed=100 + i)
        gx = torch.Generator().manual_seed(200 + i)
        with torch.no_grad():
            for n in ["wq", "wk", "wv", "wo"]:
                getattr(blk, n).weight.copy_(w[n])
            blk.q_norm.weight.copy_(w["q_norm"])
            blk.k_norm.weight.copy_(w["k_norm"])
            x = torch.randn(1, seq, dim, generator=gx).bfloat16().float()
            mask = torch.ones(1, seq, dtype=torch.bool)
            third = hd // 2 // 3 * 2
            axes = (hd - 2 * third, third, third)
            emb3 = L.RopeEmbedder(theta=10000.0, axes_dims=axes, axes_lens=(1, 64, 64))
            ids3 = torch.zeros(1, seq, 3, dtype=torch.int32)
            ids3[0, :, 1] = torch.arange(seq) // side
            ids3[0, :, 2] = torch.arange(seq) % side
            f3 = emb3(ids3)
            y = blk(x, mask, f3)
        ja[f"{tag}_x_bf16"] = bf16_bits(x.bfloat16())
        ja[f"{tag}_freqs"] = torch.view_as_real(f3).numpy()
        ja[f"{tag}_y"] = y.numpy()
        ja[f"{tag}_meta"] = np.array([dim, heads, kvh, seq, 100 + i], dtype=np.int64)
        ja[f"{tag}_wsum"] = np.array([float(w[n].double().sum()) for n in ["wq", "wk", "wv", "wo", "q_norm", "k_norm"]])
    np.savez_compressed(OUT_JATTN, **ja)
    print(f"wrote {OUT_JATTN} ({OUT_JATTN.stat().st_size} bytes, {len(ja)} arrays)")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py <path of the quantfun2 source tree>")
    main(sys.argv[1])
