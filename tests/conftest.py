"""Test configuration: the `gpu` marker (tests that need an sm_100 GPU, run on the B200 box
with `-m gpu`), golden-vector access and shared helpers. CPU tests (`-m "not gpu"`) check the
oracle against the reference's golden vectors, the host logic and the C-ABI library's exports."""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest
import torch

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = Path(__file__).resolve().parent / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 (B200) GPU and the built library")


def has_b200() -> bool:
    return torch.cuda.is_available() and torch.cuda.get_device_capability(0) == (10, 0)


def pytest_collection_modifyitems(config, items):
    if has_b200():
        return
    skip = pytest.mark.skip(reason="needs an sm_100 GPU")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def golden():
    with np.load(GOLDEN / "int8_golden.npz") as z:
        return {k: z[k] for k in z.files}


def bits_to_torch(bits: np.ndarray, dtype: torch.dtype) -> torch.Tensor:
    """uint16 bit patterns -> a bf16 / fp16 tensor."""
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(dtype)


def torch_to_bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


DTAG = {torch.bfloat16: "bf16", torch.float16: "f16"}
