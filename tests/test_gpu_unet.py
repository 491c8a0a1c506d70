"""SDXL-style UNet on the W8A8 linears and INT8 attention against the REFERENCE's own UNet
(tests/golden/unet_tiny.npz, made by make_unet_golden.py from src/diffucore/models/unet.py with the
reference's W8A8 torch-op linears, ConvRot group 0, and exact SDPA; bf16).

With exact attention the only differences left are cuDNN / CUDA GroupNorm, LayerNorm and SDPA
against their CPU counterparts (the int8 codes of a linear are bit-exact given the same input);
with INT8 self-attention (head dim 64, the reference falls back to SDPA there) its quantization
error adds on top.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from diffucore_b200 import _attention, unet
from tests.conftest import GOLDEN, bits_to_torch

pytestmark = pytest.mark.gpu
CFG = dict(model_channels=32, channel_mult=(1, 2), transformer_depth=(0, 1), num_head_channels=64, context_dim=64,
           adm_in_channels=32, use_linear_in_transformer=True)


def _fixture():
    with np.load(GOLDEN / "unet_tiny.npz") as z:
        return {k: z[k] for k in z.files}


@pytest.mark.parametrize("backend", ["sdpa", "int8_turing"])
def test_unet_matches_reference_fixture(backend):
    fx = _fixture()
    model = unet.UNetModel(unet.UNetConfig(**CFG))
    unet.init_random_(model, seed=0, device="cpu", dtype=torch.bfloat16)
    assert sorted(model.int8_linear_names()) == sorted(fx["names"])
    model = model.cuda()
    unet.quantize_linears(model, model.int8_linear_names(), "cuda", group=0)
    _attention.set_attention_backend(model, backend)
    assert model.input_blocks[4][1].transformer_blocks[0].attn2.attn_backend == "sdpa"   # cross stays exact
    x = bits_to_torch(fx["x"], torch.bfloat16).cuda()
    ctx = bits_to_torch(fx["ctx"], torch.bfloat16).cuda()
    y = bits_to_torch(fx["y"], torch.bfloat16).cuda()
    with torch.no_grad():
        for i, t in enumerate(fx["times"]):
            eps = model(x, torch.full((2,), float(t), device="cuda"), ctx, y).float().cpu()
            want = bits_to_torch(fx[f"eps_t{i}"], torch.bfloat16).float()
            assert torch.isfinite(eps).all()
            cos = F.cosine_similarity(eps.flatten().double(), want.flatten().double(), dim=0).item()
            rel = ((eps - want).norm() / want.norm()).item()
            # Whole-model bar (as for the full-width FLUX check): CPU and GPU convolutions,
            # GroupNorm and SDPA differ in the last bf16 bit and each int8 requantization spreads
            # that to neighbouring codes, so outputs of magnitude ~3 land a bf16 ulp or two apart
            # (measured with exact attention: max-abs 0.043, cosine 0.99983).
            if backend == "sdpa":
                assert cos >= 0.999 and rel < 3e-2, (cos, rel)
            else:
                assert cos >= 0.998 and rel < 5e-2, (cos, rel)


def test_sdxl_unet_full_size_step():
    """BASELINE config 3 shapes: SDXL UNet (320/640/1280, depth 0/2/10, head dim 64, context
    2048), CFG batch 2 at 1024^2 (latent 4 x 128 x 128): one Euler step runs, INT8 self-attention
    at 4096 and 1024 tokens, finite output."""
    model = unet.build_sdxl_unet(seed=0, device="cuda")
    g = torch.Generator(device="cuda").manual_seed(0)
    x = torch.randn(1, 4, 128, 128, generator=g, device="cuda").half()
    ctx = torch.randn(2, 77, 2048, generator=g, device="cuda").half()
    y = torch.randn(2, 2816, generator=g, device="cuda").half()
    out = unet.euler_cfg_sample(model, x, ctx, y, steps=2)
    assert out.shape == x.shape and torch.isfinite(out).all()
