"""Generates ``flux_tiny.npz``: the REFERENCE's own FLUX DiT (diffucore 0.2.4,
``src/diffucore/models/flux_dit.py``) run on CPU with its W8A8 linears on the torch-op path
(``src/diffucore/models/_int8.py``) and the exact SDPA attention backend, on a small FLUX.1
configuration with seeded random weights and inputs.

Run in a checkout that has the reference sources (it is never run by the tests):
    PYTHONPATH=<reference>/src python tests/golden/make_flux_golden.py

Weights come from ``diffucore_b200.flux.init_random_`` (seeded, by parameter name, so this
package's ``Flux`` gets the same values); every block linear is then quantized with the
reference's ``Int8Linear.from_linear`` for ConvRot group 0 and, separately, group 256.
Stored (16-bit tensors as uint16 bit patterns): the inputs, and for each group the velocity of
two forward calls (t = 0.75 and t = 0.25).
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))

from diffucore.models import _int8 as ref_int8          # noqa: E402  the reference
from diffucore.models import flux_dit as ref_flux       # noqa: E402

from diffucore_b200 import flux as ours                 # noqa: E402  (weights init, ids, config)

CFG = dict(in_channels=64, context_in_dim=64, vec_in_dim=32, hidden_size=256, mlp_ratio=4.0, num_heads=2,
           depth=2, depth_single_blocks=2, axes_dim=(16, 56, 56), theta=10_000, qkv_bias=True,
           guidance_embed=False)
N_TXT, GRID_H, GRID_W = 40, 8, 12          # 40 text + 96 image tokens = 136
TIMES = (0.75, 0.25)


def bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16).copy()


def inputs():
    g = torch.Generator().manual_seed(7)
    img = torch.randn(1, GRID_H * GRID_W, CFG["in_channels"], generator=g).to(torch.bfloat16)
    txt = torch.randn(1, N_TXT, CFG["context_in_dim"], generator=g).to(torch.bfloat16)
    y = torch.randn(1, CFG["vec_in_dim"], generator=g).to(torch.bfloat16)
    return img, txt, y


def reference_model(group: int):
    model = ref_flux.Flux(ref_flux.FluxConfig(**CFG))
    ours.init_random_(model, seed=0, device="cpu")
    names = [n for n, m in model.named_modules() if isinstance(m, torch.nn.Linear)
             and (".img_attn." in n or ".txt_attn." in n or "_mlp." in n or n.endswith("linear1")
                  or n.endswith("linear2")) and n.startswith(("double_blocks", "single_blocks"))]
    for name in names:
        parent, attr = ref_int8._parent(model, name)
        setattr(parent, attr, ref_int8.Int8Linear.from_linear(getattr(parent, attr), group, "cpu"))
    return model.eval(), names


def main() -> None:
    assert not ref_int8._fast(torch.zeros(1)), "the reference must run its torch-op path"
    img, txt, y = inputs()
    iid = ours.img_ids(GRID_H * 2, GRID_W * 2, 2)
    tid = ours.txt_ids(N_TXT)
    out = {"img": bits(img), "txt": bits(txt), "y": bits(y), "img_ids": iid.numpy(), "txt_ids": tid.numpy(),
           "times": np.array(TIMES, dtype=np.float32)}
    for group in (0, 256):
        model, names = reference_model(group)
        with torch.no_grad():
            for i, t in enumerate(TIMES):
                ts = torch.full((1,), t, dtype=torch.bfloat16)
                v = model(img, iid, txt, tid, ts, y)
                out[f"v_g{group}_t{i}"] = bits(v[0])
        out[f"names_g{group}"] = np.array(names)
    np.savez_compressed(HERE / "flux_tiny.npz", **out)
    print({k: v.shape for k, v in out.items()})


if __name__ == "__main__":
    main()
