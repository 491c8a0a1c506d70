"""Builds the reference's own INT8 attention kernels (diffucore 0.2.4,
``src/diffucore/kernels/int8_attn_sm80.cu``) from its source where it lies, with the flags the
reference's JIT build uses on a capability-10.0 GPU (``_attention.py:97-103``:
``-O3 -std=c++20 -gencode=arch=compute_100,code=sm_100``), plus ``oracle/ref_attn_shim.cu`` which
exposes the prep kernels' outputs. Output goes to ``oracle/_ref/`` only (git-ignored; it travels
to the GPU box with the snapshot). TEST INFRASTRUCTURE ONLY.

Usage (where the reference checkout exists):  python -m oracle.build_ref [<reference root>]
On the GPU box, :func:`load` imports the prebuilt module without the sources.
"""

from __future__ import annotations

import importlib.util
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_ref"
NAME = "dc_ref_attn_sm100"


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


def available() -> bool:
    return (OUT / f"{NAME}.so").exists()


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


if __name__ == "__main__":
    print(build(sys.argv[1] if len(sys.argv) > 1 else "/root/reference"))
