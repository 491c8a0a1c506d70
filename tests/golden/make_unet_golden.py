"""Generates ``unet_tiny.npz``: the REFERENCE's own SD/SDXL UNet (diffucore 0.2.4,
``src/diffucore/models/unet.py``) run on CPU with its W8A8 attention / feed-forward linears on the
torch-op path (``src/diffucore/models/_int8.py``, ConvRot group 0) and exact SDPA attention, on a
small SDXL-style configuration with seeded weights (``diffucore_b200.unet.init_random_``, by
parameter name) and seeded inputs, in bf16.

Run in a checkout that has the reference sources (it is never run by the tests):
    PYTHONPATH=<reference>/src python tests/golden/make_unet_golden.py
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))

from diffucore.models import _int8 as ref_int8          # noqa: E402  the reference
from diffucore.models import unet as ref_unet           # noqa: E402

from diffucore_b200 import unet as ours                 # noqa: E402  (weights init, names)

CFG = dict(model_channels=32, channel_mult=(1, 2), transformer_depth=(0, 1), num_head_channels=64, context_dim=64,
           adm_in_channels=32, use_linear_in_transformer=True)
TIMES = (999.0, 500.0)


def bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16).copy()


def main() -> None:
    assert not ref_int8._fast(torch.zeros(1)), "the reference must run its torch-op path"
    model = ref_unet.UNetModel(ref_unet.UNetConfig(**CFG))
    ours.init_random_(model, seed=0, device="cpu", dtype=torch.bfloat16)
    names = ours.UNetModel(ours.UNetConfig(**CFG)).int8_linear_names()
    for name in names:
        parent, attr = ref_int8._parent(model, name)
        setattr(parent, attr, ref_int8.Int8Linear.from_linear(getattr(parent, attr), 0, "cpu"))
    model.eval()
    g = torch.Generator().manual_seed(11)
    x = torch.randn(2, 4, 16, 16, generator=g).to(torch.bfloat16)
    ctx = torch.randn(2, 77, 64, generator=g).to(torch.bfloat16)
    y = torch.randn(2, 32, generator=g).to(torch.bfloat16)
    out = {"x": bits(x), "ctx": bits(ctx), "y": bits(y), "times": np.array(TIMES, dtype=np.float32),
           "names": np.array(names)}
    with torch.no_grad():
        for i, t in enumerate(TIMES):
            eps = model(x, torch.full((2,), t), ctx, y)
            out[f"eps_t{i}"] = bits(eps)
    np.savez_compressed(HERE / "unet_tiny.npz", **out)
    print({k: v.shape for k, v in out.items()})


if __name__ == "__main__":
    main()
