"""Generates the golden vectors in this directory by running the REFERENCE's own code
(diffucore 0.2.4, ``src/diffucore/models/_int8.py``, torch-op path, CPU) on seeded inputs.

Run in a checkout that has the reference sources (it is never run by the tests):
    PYTHONPATH=<reference>/src python tests/golden/make_golden.py

Outputs
  int8_golden.npz    small cases: quantize_activation (group 0 / 256, bf16 / fp16), int_mm, rescale,
                     Int8Linear.from_linear + forward, int8_mlp, zero / tiny rows, M <= 16 padding.
  config1_sha256.json  SHA-256 of the reference's int8 codes, scales and bf16 output of
                     BASELINE config 1 (X [4096, 3072] ~ N(0,1), W [3072, 3072] ~ N(0,0.02),
                     bias ~ N(0,0.01), drawn in that order from torch.Generator seed 0, group 0),
                     so the full-size GPU result can be checked bit for bit without shipping 25 MB.
16-bit tensors are stored as their uint16 bit patterns.
"""

from __future__ import annotations

import hashlib
import json
from pathlib import Path

import numpy as np
import torch
import torch.nn as nn
import torch.nn.functional as F

from diffucore.models import _int8 as ref  # the reference implementation

HERE = Path(__file__).resolve().parent


def bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16).copy()


def sha(a: torch.Tensor) -> str:
    t = a.contiguous()
    if t.dtype in (torch.bfloat16, torch.float16):
        t = t.view(torch.int16)
    return hashlib.sha256(t.numpy().tobytes()).hexdigest()


def config1_inputs():
    g = torch.Generator().manual_seed(0)
    x = torch.randn(4096, 3072, generator=g).to(torch.bfloat16)
    w = (torch.randn(3072, 3072, generator=g) * 0.02).to(torch.bfloat16)
    b = (torch.randn(3072, generator=g) * 0.01).to(torch.bfloat16)
    return x, w, b


def main() -> None:
    assert not ref._fast(torch.zeros(1)), "the golden vectors come from the reference's torch-op path"
    out: dict[str, np.ndarray] = {}
    g = torch.Generator().manual_seed(1234)

    # quantize_activation: (M, K), dtype, group
    for name, (M, K), dt, group in (("qa_bf16_g0", (37, 512), torch.bfloat16, 0),
                                     ("qa_bf16_g256", (21, 768), torch.bfloat16, 256),
                                     ("qa_f16_g0", (19, 320), torch.float16, 0),
                                     ("qa_f16_g256", (9, 512), torch.float16, 256)):
        x = (torch.randn(M, K, generator=g) * 3).to(dt)
        x[1, :] = 0                                    # all-zero row: scale clamps to 1e-30
        x[2, 5] = 1e-3                                 # single tiny value
        q, s = ref.quantize_activation(x, group)
        out[f"{name}_x"], out[f"{name}_q"], out[f"{name}_s"] = bits(x), q.numpy(), s.numpy()

    # int_mm: includes M <= 16 (the reference pads to 32) and the bit-exact test shapes' K
    for name, (m, n, k) in (("imm_small", (3, 96, 256)), ("imm_mid", (33, 160, 512))):
        qa = torch.randint(-127, 128, (m, k), generator=g, dtype=torch.int8)
        wa = torch.randint(-127, 128, (n, k), generator=g, dtype=torch.int8)
        out[f"{name}_q"], out[f"{name}_w"], out[f"{name}_acc"] = qa.numpy(), wa.numpy(), ref.int_mm(qa, wa).numpy()

    # rescale with the reference test's scale ranges (tests/test_int8.py:181), bf16/fp16, with and
    # without bias
    for dt, tag in ((torch.bfloat16, "bf16"), (torch.float16, "f16")):
        acc = torch.randint(-2_000_000, 2_000_000, (29, 136), generator=g, dtype=torch.int32)
        sx, sw = torch.rand(29, generator=g) * 1e-2, torch.rand(136, generator=g) * 1e-3
        bias = (torch.randn(136, generator=g) * 0.1).to(dt)
        out[f"rs_{tag}_acc"], out[f"rs_{tag}_sx"], out[f"rs_{tag}_sw"] = acc.numpy(), sx.numpy(), sw.numpy()
        out[f"rs_{tag}_bias"] = bits(bias)
        out[f"rs_{tag}_y"] = bits(ref.rescale(acc, sx, sw, None, dt))
        out[f"rs_{tag}_yb"] = bits(ref.rescale(acc, sx, sw, bias, dt))

    # Int8Linear: from_linear (weights) + forward, group 0 and 256, with bias
    for tag, group, dt in (("lin_g0_bf16", 0, torch.bfloat16), ("lin_g256_bf16", 256, torch.bfloat16),
                           ("lin_g0_f16", 0, torch.float16)):
        torch.manual_seed(7)
        lin = nn.Linear(512, 192, bias=True).to(dt)
        with torch.no_grad():
            lin.weight.copy_((torch.randn(192, 512, generator=g) * 0.02).to(dt))
            lin.bias.copy_((torch.randn(192, generator=g) * 0.01).to(dt))
        layer = ref.Int8Linear.from_linear(lin, group)
        x = torch.randn(2, 40, 512, generator=g).to(dt)
        y = layer(x)
        out[f"{tag}_w"], out[f"{tag}_b"], out[f"{tag}_x"] = bits(lin.weight.detach()), bits(lin.bias.detach()), bits(x)
        out[f"{tag}_wq"], out[f"{tag}_ws"], out[f"{tag}_y"] = layer.weight.numpy(), layer.scale.numpy(), bits(y)
        out[f"{tag}_float"] = lin(x).detach().float().numpy()

    # int8_mlp (torch-op path = l2(gelu(l1(x))), erf GELU), bias-free as in Anima
    l1 = ref.Int8Linear.from_linear(nn.Linear(256, 512, bias=False).to(torch.bfloat16), 0)
    l2 = ref.Int8Linear.from_linear(nn.Linear(512, 256, bias=False).to(torch.bfloat16), 0)
    x = torch.randn(3, 50, 256, generator=g).to(torch.bfloat16)
    out["mlp_x"], out["mlp_y"] = bits(x), bits(ref.int8_mlp(x, l1, l2))
    out["mlp_l1q"], out["mlp_l1s"] = l1.weight.numpy(), l1.scale.numpy()
    out["mlp_l2q"], out["mlp_l2s"] = l2.weight.numpy(), l2.scale.numpy()
    out["mlp_h"] = bits(F.gelu(l1(x)))

    # signs of the normalised 256-Hadamard (every entry is +-1/16)
    out["hadamard256_sign"] = torch.sign(ref._hadamard(256, "cpu")).to(torch.int8).numpy()
    assert torch.equal(ref._hadamard(256, "cpu").abs(), torch.full((256, 256), 0.0625))

    np.savez_compressed(HERE / "int8_golden.npz", **out)

    # config 1 at full size: hashes of the reference's codes / scales / output
    x, w, b = config1_inputs()
    lin = nn.Linear(3072, 3072, bias=True).to(torch.bfloat16)
    with torch.no_grad():
        lin.weight.copy_(w)
        lin.bias.copy_(b)
    layer = ref.Int8Linear.from_linear(lin, 0)
    qx, sx = ref.quantize_activation(x, 0)
    y = layer(x)
    meta = {
        "inputs": "torch.Generator().manual_seed(0); X=randn(4096,3072), W=randn(3072,3072)*0.02, "
                  "b=randn(3072)*0.01, each .to(bfloat16), drawn in that order; group 0",
        "x_sha256": sha(x), "w_sha256": sha(w), "b_sha256": sha(b),
        "wq_sha256": sha(layer.weight), "ws_sha256": sha(layer.scale),
        "qx_sha256": sha(qx), "sx_sha256": sha(sx), "y_sha256": sha(y),
        "acc_sha256": sha(ref.int_mm(qx, layer.weight)),
    }
    (HERE / "config1_sha256.json").write_text(json.dumps(meta, indent=1) + "\n")
    print("wrote", sorted(out)[:5], "...", len(out), "arrays; config1 hashes")


if __name__ == "__main__":
    main()
