"""On-disk prepared weights (xpu_kernels.int8.checkpoint), on CPU.

The weights are prepared by the CPU oracle (the restatement of the
reference's prepare_weight), saved, loaded and validated; malformed layers are
rejected with the rule they break.
"""

import numpy as np
import pytest
import torch

from oracle import convrot_oracle as O
from xpu_kernels.int8 import checkpoint as C


def _layer(n=32, k=256, seed=0, bias=True):
    rng = np.random.default_rng(seed)
    w = O.round_bf16((rng.standard_normal((n, k)) * 0.02).astype(np.float32))
    w8, ws = O.prepare_weight(w)
    b = torch.from_numpy((rng.standard_normal(n) * 0.01).astype(np.float32)) if bias else None
    return torch.from_numpy(w8), torch.from_numpy(ws), b


def test_round_trip(tmp_path):
    layers = {"q": _layer(32, 256, 1), "mlp.up": _layer(64, 512, 2, bias=False)}
    path = tmp_path / "w.pt"
    C.save_int8_linear(path, layers)
    got = C.load_int8_linear(path)
    assert set(got) == {"q", "mlp.up"}
    for name, (w8, ws, b) in layers.items():
        g8, gs, gb = got[name]
        assert torch.equal(g8, w8) and torch.equal(gs, ws)
        assert (gb is None) == (b is None) and (b is None or torch.equal(gb, b))


def test_scale_shapes_accepted():
    w8, ws, _ = _layer()
    C.validate_weight(w8, ws)                    # [N]
    C.validate_weight(w8, ws.reshape(-1, 1))     # [N, 1]
    C.validate_weight(w8, torch.tensor(0.01))    # scalar


@pytest.mark.parametrize("bad,rule", [
    (lambda w8, ws: (w8.float(), ws), "int8"),
    (lambda w8, ws: (w8[:, :200], ws), "multiple of the ConvRot group"),
    (lambda w8, ws: (w8[:24], ws[:24]), "multiple of 16"),
    (lambda w8, ws: (torch.full_like(w8, -128), ws), "-128"),
    (lambda w8, ws: (w8, ws.double()), "fp32"),
    (lambda w8, ws: (w8, ws[:5]), "[N]"),
    (lambda w8, ws: (w8, -ws), "positive"),
    (lambda w8, ws: (w8, ws * float("inf")), "finite"),
])
def test_malformed_layers_are_rejected(bad, rule):
    w8, ws, _ = _layer()
    a, b = bad(w8, ws)
    with pytest.raises(ValueError, match=rule.replace("[", r"\[").replace("]", r"\]")):
        C.validate_weight(a, b, "layer0")


def test_loading_requires_the_format_entry(tmp_path):
    w8, ws, b = _layer()
    path = tmp_path / "plain.pt"
    torch.save({"fc.weight": w8, "fc.weight_scale": ws}, path)
    with pytest.raises(ValueError, match="not a ConvRot INT8 checkpoint"):
        C.load_int8_linear(path)
    assert set(C.load_int8_linear(path, require_meta=False)) == {"fc"}
    torch.save({C.META_KEY: {"format": "int8-plain", "group": 256}, "fc.weight": w8,
                "fc.weight_scale": ws}, path)
    with pytest.raises(ValueError, match="format"):
        C.load_int8_linear(path)
    torch.save({C.META_KEY: dict(C.FORMAT), "fc.weight": w8}, path)
    with pytest.raises(ValueError, match="no weight_scale"):
        C.load_int8_linear(path)


@pytest.mark.gpu
def test_prepared_state_dict_round_trip_on_gpu(tmp_path):
    """bf16 state dict -> prepare_weight on the GPU -> file -> linear: the loaded
    layer gives the same output as the freshly prepared one, and the prepared
    weight is the oracle's."""
    import xpu_kernels
    g = torch.Generator().manual_seed(3)
    sd = {"a.weight": (torch.randn(64, 512, generator=g) * 0.02).to(torch.bfloat16),
          "a.bias": torch.randn(64, generator=g) * 0.01,
          "odd.weight": torch.randn(10, 512, generator=g)}    # N % 16: skipped
    layers = C.prepare_state_dict(sd, device="cuda")
    assert set(layers) == {"a"}
    path = tmp_path / "p.pt"
    C.save_int8_linear(path, layers)
    got = C.load_int8_linear(path, device="cuda")
    w8r, wsr = O.prepare_weight(sd["a.weight"].view(torch.int16).numpy().view(np.uint16))
    assert np.array_equal(got["a"][0].cpu().numpy(), w8r)
    x = torch.randn(33, 512, generator=g).to(torch.bfloat16).cuda()
    y1 = xpu_kernels.linear(x, *layers["a"])
    y2 = xpu_kernels.linear(x, *got["a"])
    assert torch.equal(y1.view(torch.int16), y2.view(torch.int16))
