"""GPU: quantize-on-load from safetensors (create_quantized_model_from_safetensors, the
mirror of src/pipeline.py:289-340) gives bit-identical codes and scales to quantizing the
loaded model with quantize_model, and the same outputs."""
import copy

import pytest
import torch

pytestmark = pytest.mark.gpu


class _Block(torch.nn.Module):
    def __init__(self, dim=256):
        super().__init__()
        self.norm = torch.nn.Parameter(torch.rand(dim) + 0.5)
        self.attn = torch.nn.ModuleDict({"wq": torch.nn.Linear(dim, dim, bias=False),
                                         "wo": torch.nn.Linear(dim, dim, bias=True)})
        self.mlp = torch.nn.Sequential(torch.nn.Linear(dim, 512), torch.nn.GELU(), torch.nn.Linear(512, dim))

    def forward(self, x):
        h = x * self.norm
        return self.attn["wo"](self.attn["wq"](h)) + self.mlp(h)


class _Model(torch.nn.Module):
    def __init__(self):
        super().__init__()
        self.embed = torch.nn.Linear(64, 256)
        self.blocks = torch.nn.ModuleList([_Block(), _Block()])

    def forward(self, x):
        x = self.embed(x)
        for b in self.blocks:
            x = x + b(x)
        return x


@pytest.mark.parametrize("qname", ["qint8", "qfloat8", "qfloat8_w8a8"])
def test_safetensors_quantize_on_load_matches_quantize_model(cuda, tmp_path, qname):
    from safetensors.torch import save_file

    from quantfun2_b200 import quant
    from quantfun2_b200.loader import create_quantized_model_from_safetensors

    q = getattr(quant, qname)
    torch.manual_seed(0)
    m = _Model()
    path = tmp_path / "model.safetensors"
    save_file({k: v.contiguous() for k, v in m.state_dict().items()}, str(path))
    # like the reference's, quantize_model moves only the converted linears to the device
    ref = quant.quantize_model(copy.deepcopy(m), q, device="cuda", quantization_device="cuda").to(cuda)
    with torch.device("meta"):
        meta = _Model()
    got = create_quantized_model_from_safetensors(meta, path, device="cuda", quantization_device="cuda", dtype=q)
    assert list(got.state_dict().keys()) == list(m.state_dict().keys())
    lin_names = [n for n, mod in ref.named_modules() if isinstance(mod, torch.nn.Linear)]
    assert len(lin_names) == 9
    for n in lin_names:
        a, b = ref.get_submodule(n).weight, got.get_submodule(n).weight
        assert isinstance(b, quant.QuantizedWeight)
        assert torch.equal(a.codes, b.codes) and torch.equal(a.scale, b.scale), n
        ba, bb = ref.get_submodule(n).bias, got.get_submodule(n).bias
        assert (ba is None and bb is None) or torch.equal(ba, bb), n
    for i in range(2):
        assert torch.equal(ref.blocks[i].norm, got.blocks[i].norm)
    act = q.supported_dtypes[0]
    x = torch.randn(3, 100, 64, device=cuda).to(act)
    assert torch.equal(ref(x), got(x))
