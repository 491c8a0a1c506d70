"""ComfyUI ``int8_tensorwise`` checkpoints, the on-disk format of the W8A8 layers, load into the
FLUX and SDXL backbones (reference src/diffucore/models/_int8.py:453-481 and the loader sequence
src/diffucore/bundle.py:301-305). CPU only.

A model whose block linears were quantized in memory is written out in the int8_tensorwise layout
(int8 ``weight``, fp32 ``weight_scale``, ``comfy_quant`` JSON tag), read back through
``from_state_dict`` (meta build, ``int8_layers`` + ``adopt_int8_layers``, strict load), and must
carry the same buffers; the FLUX runner (kernels restated in torch) gives the same velocity.
"""

from __future__ import annotations

import json

import pytest
import torch

from diffucore_b200 import _int8, flux, unet
from tests.flux_torch_ops import TorchOps

FLUX_CFG = dict(in_channels=64, context_in_dim=64, vec_in_dim=32, hidden_size=256, mlp_ratio=4.0, num_heads=2,
                depth=1, depth_single_blocks=1)
UNET_CFG = dict(model_channels=32, channel_mult=(1, 2), transformer_depth=(0, 1), num_head_channels=64,
                context_dim=64, adm_in_channels=32, use_linear_in_transformer=True)


def to_int8_tensorwise(model: torch.nn.Module) -> dict:
    """State dict with every Int8Linear written the way ComfyUI stores int8_tensorwise layers."""
    sd = {}
    int8 = {n: m for n, m in model.named_modules() if isinstance(m, _int8.Int8Linear)}
    for key, t in model.state_dict().items():
        layer, _, leaf = key.rpartition(".")
        if layer in int8 and leaf == "scale_bits":
            sd[layer + ".weight_scale"] = t.view(torch.float32).clone()
            meta = {"format": "int8_tensorwise", "convrot": int8[layer].group > 0,
                    "convrot_groupsize": int8[layer].group}
            sd[layer + ".comfy_quant"] = torch.tensor(list(json.dumps(meta).encode()), dtype=torch.uint8)
        else:
            sd[key] = t.clone()
    return sd


@pytest.mark.parametrize("group", [0, 256])
def test_flux_int8_tensorwise_round_trip(group):
    cfg = flux.FluxConfig(**FLUX_CFG)
    model = flux.Flux(cfg)
    flux.init_random_(model, seed=4, device="cpu")
    flux.quantize_linears(model, model.block_linear_names(), "cpu", group=group)
    sd = to_int8_tensorwise(model)
    assert sum(k.endswith(".comfy_quant") for k in sd) == len(model.block_linear_names())
    loaded = flux.from_state_dict(sd, cfg, device="cpu")
    a, b = model.state_dict(), loaded.state_dict()
    assert a.keys() == b.keys()
    assert all(torch.equal(a[k], b[k]) for k in a)
    assert all(loaded.get_submodule(n).group == group for n in model.block_linear_names())

    g = torch.Generator().manual_seed(2)
    img = torch.randn(48, 64, generator=g).to(torch.bfloat16)
    txt = torch.randn(16, 64, generator=g).to(torch.bfloat16)
    y = torch.randn(1, 32, generator=g).to(torch.bfloat16)
    t = torch.full((1,), 0.5, dtype=torch.bfloat16)
    outs = []
    for m in (model, loaded):
        r = flux.FluxRunner(m, 16, 48, device="cpu", ops=TorchOps())
        r.set_positions(flux.img_ids(12, 16, 2), flux.txt_ids(16))
        outs.append(r.forward(img, txt, t, y))
    assert torch.equal(outs[0], outs[1])


def test_unet_int8_tensorwise_round_trip():
    cfg = unet.UNetConfig(**UNET_CFG)
    model = unet.UNetModel(cfg)
    unet.init_random_(model, seed=5, device="cpu", dtype=torch.bfloat16)
    names = model.int8_linear_names()
    unet.quantize_linears(model, names, "cpu", group=0)
    loaded = unet.from_state_dict(to_int8_tensorwise(model), cfg, device="cpu")
    a, b = model.state_dict(), loaded.state_dict()
    assert a.keys() == b.keys() and all(torch.equal(a[k], b[k]) for k in a)
    assert sorted(n for n, m in loaded.named_modules() if isinstance(m, _int8.Int8Linear)) == sorted(names)


def test_plain_checkpoint_loads_without_adoption():
    cfg = flux.FluxConfig(**FLUX_CFG)
    model = flux.Flux(cfg)
    flux.init_random_(model, seed=6, device="cpu")
    loaded = flux.from_state_dict(model.state_dict(), cfg, device="cpu")
    assert not any(isinstance(m, _int8.Int8Linear) for m in loaded.modules())
    assert all(torch.equal(model.state_dict()[k], v) for k, v in loaded.state_dict().items())


def test_unsupported_quantized_format_is_refused():
    cfg = flux.FluxConfig(**FLUX_CFG)
    model = flux.Flux(cfg)
    sd = model.state_dict()
    sd["double_blocks.0.img_attn.qkv.comfy_quant"] = torch.tensor(list(b'{"format": "float8_e4m3fn"}'),
                                                                  dtype=torch.uint8)
    with pytest.raises(ValueError, match="int8_tensorwise"):
        flux.from_state_dict(sd, cfg, device="cpu")
