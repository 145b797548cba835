"""Loader of the reference JointAttention golden cases (tests/golden/ref_jattn.npz)."""
import numpy as np

from oracle.numerics import bf16_bits_to_f32


def jattn_case(tag):
    """Inputs, weights and reference output of a tests/golden/ref_jattn.npz case; the weights
    are rebuilt from their seed with the generating script's own function."""
    import importlib.util
    from pathlib import Path

    root = Path(__file__).resolve().parent / "golden"
    spec = importlib.util.spec_from_file_location("make_golden", root / "make_golden.py")
    mg = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mg)
    g = np.load(root / "ref_jattn.npz")
    dim, heads, kvh, seq, seed = [int(v) for v in g[f"{tag}_meta"]]
    w = mg.jattn_weights(dim, heads, kvh, seed)
    sums = [float(w[n].double().sum()) for n in ["wq", "wk", "wv", "wo", "q_norm", "k_norm"]]
    np.testing.assert_allclose(sums, g[f"{tag}_wsum"], rtol=0, atol=1e-9)  # same generator stream
    return dict(dim=dim, heads=heads, kvh=kvh, seq=seq, w={k: v.numpy() for k, v in w.items()},
                x=bf16_bits_to_f32(g[f"{tag}_x_bf16"]), freqs=g[f"{tag}_freqs"], y=g[f"{tag}_y"])
