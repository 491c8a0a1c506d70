"""Builds and stages the reference's own implementation of the hot path as a checker and GPU bar —
TEST INFRASTRUCTURE ONLY (nothing in ``diffucore_b200`` loads any of it).

* :func:`build` compiles the reference's INT8 attention kernels (diffucore 0.2.4,
  ``src/diffucore/kernels/int8_attn_sm80.cu``) from their source where it lies, with the flags the
  reference's JIT build uses on a capability-10.0 GPU (``_attention.py:97-103``:
  ``-O3 -std=c++20 -gencode=arch=compute_100,code=sm_100``), plus ``oracle/ref_attn_shim.cu`` which
  exposes the prep kernels' outputs.
* :func:`stage_python` copies the reference's ``src/diffucore/models/_int8.py`` unchanged (its
  Triton ``_rot_quant_kernel`` / ``_rescale_kernel`` and torch-op GPU path, ``_int8.py:299-323``,
  ``:399-417``) so that it can be imported on the GPU box, where the reference checkout is absent;
  and, unchanged, the model modules the drop-in test runs (``flux_dit.py``, ``anima_dit.py`` and the
  modules they import) as a package ``diffucore.models`` under ``oracle/_ref/refpkg`` (its two
  ``__init__.py`` are written empty there, since the reference's own import its whole pipeline
  stack, which the test does not use).

Output goes to ``oracle/_ref/`` only (git-ignored; it travels to the GPU box with the snapshot).

Usage (where the reference checkout exists):
    python -m oracle.build_ref [<reference root>]
The root defaults to the environment variable ``DIFFUCORE_REFERENCE``, else to a checkout named
``reference`` beside this repository.
"""

from __future__ import annotations

import importlib.util
import os
import shutil
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_ref"
NAME = "dc_ref_attn_sm100"
INT8_STAGED = OUT / "ref_int8.py"
REF_PKG = OUT / "refpkg"
REF_MODELS = ("_int8.py", "_attention.py", "_fused.py", "_norm.py", "flux_dit.py", "anima_dit.py", "llm_adapter.py")


def default_root() -> Path | None:
    """The reference checkout: ``DIFFUCORE_REFERENCE`` if set, else ``../reference`` next to this
    repository; None when neither holds the reference's sources."""
    env = os.environ.get("DIFFUCORE_REFERENCE")
    cands = [Path(env)] if env else [HERE.parent.parent / "reference"]
    for c in cands:
        if (c / "src" / "diffucore" / "kernels" / "int8_attn_sm80.cu").exists():
            return c
    return None


def build(reference_root: str | Path) -> Path:
    from torch.utils.cpp_extension import load as jit_load
    kernels = Path(reference_root) / "src" / "diffucore" / "kernels"
    if not (kernels / "int8_attn_sm80.cu").exists():
        raise FileNotFoundError(f"no int8_attn_sm80.cu under {kernels}")
    OUT.mkdir(exist_ok=True)
    jit_load(name=NAME, sources=[str(HERE / "ref_attn_shim.cu")], extra_include_paths=[str(kernels)],
             extra_cuda_cflags=["-O3", "-std=c++20", "-gencode=arch=compute_100,code=sm_100"],
             extra_cflags=["-O3", "-std=c++20"], build_directory=str(OUT), verbose=False)
    return OUT / f"{NAME}.so"


def stage_python(reference_root: str | Path) -> Path:
    """Copy the reference's ``_int8.py`` (unchanged) to ``oracle/_ref/ref_int8.py``, and the model
    modules of ``REF_MODELS`` (unchanged) to ``oracle/_ref/refpkg/diffucore/models/``."""
    models = Path(reference_root) / "src" / "diffucore" / "models"
    src = models / "_int8.py"
    if not src.exists():
        raise FileNotFoundError(f"no _int8.py at {src}")
    OUT.mkdir(exist_ok=True)
    shutil.copyfile(src, INT8_STAGED)
    pkg = REF_PKG / "diffucore" / "models"
    pkg.mkdir(parents=True, exist_ok=True)
    (REF_PKG / "diffucore" / "__init__.py").write_text("")
    (pkg / "__init__.py").write_text("")
    for name in REF_MODELS:
        shutil.copyfile(models / name, pkg / name)
    return INT8_STAGED


def available() -> bool:
    return (OUT / f"{NAME}.so").exists()


def int8_available() -> bool:
    return INT8_STAGED.exists()


def models_available() -> bool:
    return all((REF_PKG / "diffucore" / "models" / name).exists() for name in REF_MODELS)


def load():
    """The prebuilt reference module: ``mod.fwd(q, k, v, sm_scale)`` (the reference's pybind
    entry) and ``torch.ops.dcref.k_prep(k) -> [k_codes, k_scale, ksum]``."""
    import torch
    path = OUT / f"{NAME}.so"
    if not path.exists():
        raise FileNotFoundError(f"{path} is not built (run python -m oracle.build_ref <reference root>)")
    spec = importlib.util.spec_from_file_location(NAME, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    if not hasattr(torch.ops.dcref, "k_prep"):
        torch.ops.load_library(str(path))
    return mod


_int8_mod = None


def load_int8():
    """The reference's staged ``_int8.py`` as a standalone module (``quantize_activation``,
    ``int_mm``, ``rescale``, ``Int8Linear``, ...). On a CUDA tensor with Triton importable its
    ``quantize_activation`` and ``rescale`` run the reference's Triton kernels. Its fp16 fused-GEMM
    branch (``scaled_mm`` -> ``_gemm_module``) imports a sibling module and is not usable here;
    callers use bf16 or a bias, which take the int32 path as on any non-Turing GPU."""
    global _int8_mod
    if _int8_mod is None:
        if not INT8_STAGED.exists():
            raise FileNotFoundError(f"{INT8_STAGED} is not staged (run python -m oracle.build_ref <reference root>)")
        spec = importlib.util.spec_from_file_location("dc_ref_int8", INT8_STAGED)
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
        _int8_mod = mod
    return _int8_mod


if __name__ == "__main__":
    root = Path(sys.argv[1]) if len(sys.argv) > 1 else default_root()
    if root is None:
        sys.exit("reference checkout not found: pass its root or set DIFFUCORE_REFERENCE")
    print(build(root))
    print(stage_python(root))
