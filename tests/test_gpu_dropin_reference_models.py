"""The reference's own FLUX and Anima (Cosmos) model code, run on this package.

The reference's model modules (``flux_dit.py``, ``anima_dit.py`` and the modules they import),
staged unchanged into ``oracle/_ref/refpkg`` by ``oracle/build_ref.py``, import the hot path as
``diffucore.models._int8`` and ``diffucore.models._attention``. They are loaded twice: once with the
reference's own two modules there (the reference stack), once with ``diffucore_b200._int8`` and
``diffucore_b200._attention`` put in their place in ``sys.modules`` (what a maintainer does to drop
this package in). The same seeded model, with the same int8 block weights (quantized by the
reference stack, loaded into the other by ``load_state_dict``), then runs in both:

* exact attention ("sdpa") and this package's quantizer in the reference's GPU arithmetic
  (``set_quant_division("triton")``): outputs bit-identical to the reference stack's, whose int8
  linears run the reference's Triton quantizer and rescale around ``torch._int_mm``;
* INT8 attention ("int8_turing", this package's kernel; the reference's own INT8 kernel is built for
  Turing/Ampere): within the attention tolerance of the reference stack's exact-attention output.
"""

from __future__ import annotations

import importlib
import sys

import pytest
import torch

from oracle import build_ref

pytestmark = pytest.mark.gpu
DEV = "cuda"

if not build_ref.models_available():
    pytest.skip("the reference's model modules are not staged in oracle/_ref", allow_module_level=True)


def _drop_reference_modules():
    for name in [n for n in sys.modules if n == "diffucore" or n.startswith("diffucore.")]:
        del sys.modules[name]


@pytest.fixture
def stacks():
    """Loader of the two stacks; restores sys.modules and sys.path afterwards."""
    root = str(build_ref.REF_PKG)
    sys.path.insert(0, root)

    def load(ours: bool):
        _drop_reference_modules()
        importlib.import_module("diffucore.models")
        if ours:
            from diffucore_b200 import _attention, _int8
            sys.modules["diffucore.models._int8"] = _int8
            sys.modules["diffucore.models._attention"] = _attention
        mods = {n: importlib.import_module(f"diffucore.models.{n}")
                for n in ("flux_dit", "anima_dit", "_int8", "_attention")}
        return mods

    yield load
    _drop_reference_modules()
    sys.path.remove(root)


@pytest.fixture
def triton_division():
    from diffucore_b200 import _int8
    prev = _int8.quant_division()
    _int8.set_quant_division("triton")
    yield
    _int8.set_quant_division(prev)


def _close(got: torch.Tensor, want: torch.Tensor):
    g, w = got.float().flatten(), want.float().flatten()
    assert torch.isfinite(g).all()
    cos = torch.nn.functional.cosine_similarity(g.double(), w.double(), dim=0).item()
    err = (g - w).abs().max().item()
    assert cos > 0.999, cos
    assert err <= 2e-2 * max(1.0, w.abs().max().item()), err


# ----------------------------------------------------------------------------- FLUX

def _flux_names(cfg):
    names = []
    for i in range(cfg.depth):
        for s in ("img", "txt"):
            names += [f"double_blocks.{i}.{s}_attn.qkv", f"double_blocks.{i}.{s}_attn.proj",
                      f"double_blocks.{i}.{s}_mlp.0", f"double_blocks.{i}.{s}_mlp.2"]
    for i in range(cfg.depth_single_blocks):
        names += [f"single_blocks.{i}.linear1", f"single_blocks.{i}.linear2"]
    return names


def _flux_cfg(m):
    return m["flux_dit"].FluxConfig(in_channels=64, context_in_dim=64, vec_in_dim=32, hidden_size=256, num_heads=2,
                                    depth=1, depth_single_blocks=1, guidance_embed=False)


def _flux_model(m, state=None):
    fd, i8 = m["flux_dit"], m["_int8"]
    cfg = _flux_cfg(m)
    torch.manual_seed(0)
    model = fd.Flux(cfg).to(DEV, torch.float16).eval()
    i8.quantize_linears(model, _flux_names(cfg), DEV)
    if state is not None:
        model.load_state_dict(state)
    return model


def _flux_inputs():
    g = torch.Generator().manual_seed(1)
    hw = 16
    img = torch.randn(1, hw * hw, 64, generator=g).half().to(DEV)
    ids = torch.zeros(1, hw * hw, 3)
    ids[0, :, 1] = torch.arange(hw).repeat_interleave(hw).float()
    ids[0, :, 2] = torch.arange(hw).repeat(hw).float()
    txt = torch.randn(1, 64, 64, generator=g).half().to(DEV)
    y = torch.randn(1, 32, generator=g).half().to(DEV)
    t = torch.tensor([0.5], dtype=torch.float16, device=DEV)
    return img, ids.to(DEV), txt, torch.zeros(1, 64, 3, device=DEV), t, y


def test_reference_flux_on_this_package(stacks, triton_division):
    inputs = _flux_inputs()
    ref = stacks(ours=False)
    ref_model = _flux_model(ref)
    ref["_attention"].set_attention_backend(ref_model, "sdpa")
    with torch.no_grad():
        want = ref_model(*inputs)
    state = {k: v.clone() for k, v in ref_model.state_dict().items()}
    del ref_model

    ours = stacks(ours=True)
    from diffucore_b200 import _int8
    model = _flux_model(ours, state)
    assert sum(isinstance(mod, _int8.Int8Linear) for mod in model.modules()) == len(_flux_names(_flux_cfg(ours)))
    ours["_attention"].set_attention_backend(model, "sdpa")
    with torch.no_grad():
        exact = model(*inputs)
    assert torch.equal(exact, want)
    ours["_attention"].set_attention_backend(model, "int8_turing")
    with torch.no_grad():
        fast = model(*inputs)
    torch.cuda.synchronize()
    _close(fast, want)


# ----------------------------------------------------------------------------- Anima (Cosmos DiT)

def _anima_model(m, state=None):
    ad, i8 = m["anima_dit"], m["_int8"]
    cfg = ad.CosmosDiTConfig(model_channels=256, num_blocks=3, num_heads=2, head_dim=128,
                             crossattn_emb_channels=256, adaln_lora_dim=64)
    torch.manual_seed(0)
    model = ad.CosmosDiT(cfg).to(DEV, torch.float16).eval()
    i8.quantize_linears(model, ad.int8_layer_names(cfg.num_blocks), DEV)
    if state is not None:
        model.load_state_dict(state)
    return model


def test_reference_anima_on_this_package(stacks, triton_division):
    g = torch.Generator().manual_seed(2)
    x = torch.randn(1, 16, 1, 32, 32, generator=g).half().to(DEV)
    t = torch.tensor([500.0], device=DEV)
    ctx = torch.randn(1, 64, 256, generator=g).half().to(DEV)

    ref = stacks(ours=False)
    ref_model = _anima_model(ref)
    ref["_attention"].set_attention_backend(ref_model, "sdpa")
    with torch.no_grad():
        want = ref_model(x, t, ctx)
    state = {k: v.clone() for k, v in ref_model.state_dict().items()}
    del ref_model

    ours = stacks(ours=True)
    from diffucore_b200 import _int8
    model = _anima_model(ours, state)
    # block 1 of 3: q/k/v/output projections of both attentions and the two MLP linears
    assert sum(isinstance(mod, _int8.Int8Linear) for mod in model.modules()) == 10
    ours["_attention"].set_attention_backend(model, "sdpa")
    with torch.no_grad():
        exact = model(x, t, ctx)
    assert torch.equal(exact, want)
    ours["_attention"].set_attention_backend(model, "int8_turing")
    with torch.no_grad():
        fast = model(x, t, ctx)
    torch.cuda.synchronize()
    _close(fast, want)
