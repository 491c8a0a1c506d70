"""The SDXL CPU baseline's path (bench.py `sdxl_unet.cpu_baseline`: this package's UNet with every
W8A8 linear on the reference's torch-op forward, oracle/torch_ref.py `cpu_int8_linears_`, and SDPA
attention off the GPU) against the REFERENCE's own UNet run the same way (tests/golden/unet_tiny.npz,
made by make_unet_golden.py from src/diffucore/models/unet.py): the same weights, inputs and ops
on CPU give the reference's noise prediction bit for bit."""

from __future__ import annotations

import numpy as np
import torch

from diffucore_b200 import unet
from oracle.torch_ref import CpuInt8Linear, cpu_int8_linears_
from tests.conftest import GOLDEN, bits_to_torch

CFG = dict(model_channels=32, channel_mult=(1, 2), transformer_depth=(0, 1), num_head_channels=64, context_dim=64,
           adm_in_channels=32, use_linear_in_transformer=True)


def test_cpu_path_reproduces_reference_unet():
    with np.load(GOLDEN / "unet_tiny.npz") as z:
        fx = {k: z[k] for k in z.files}
    model = unet.UNetModel(unet.UNetConfig(**CFG))
    unet.init_random_(model, seed=0, device="cpu", dtype=torch.bfloat16)
    unet.quantize_linears(model, model.int8_linear_names(), "cpu", group=0)
    assert cpu_int8_linears_(model) == len(fx["names"])
    assert all(isinstance(model.get_submodule(n), CpuInt8Linear) for n in fx["names"])
    model.eval()
    x = bits_to_torch(fx["x"], torch.bfloat16)
    ctx = bits_to_torch(fx["ctx"], torch.bfloat16)
    y = bits_to_torch(fx["y"], torch.bfloat16)
    with torch.no_grad():
        for i, t in enumerate(fx["times"]):
            eps = model(x, torch.full((2,), float(t)), ctx, y)
            want = bits_to_torch(fx[f"eps_t{i}"], torch.bfloat16)
            assert torch.equal(eps, want), (eps.float() - want.float()).abs().max().item()
