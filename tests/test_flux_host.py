"""Host logic of the FLUX runner on CPU (no GPU): the runner's buffer layouts, its per-block
launch sequence and the Ulysses exchange, with every kernel replaced by the torch restatement in
``tests/flux_torch_ops.py``.

* One rank: the runner reproduces the REFERENCE's own FLUX DiT bit for bit
  (``tests/golden/flux_tiny.npz``, made by ``make_flux_golden.py`` from
  src/diffucore/models/flux_dit.py with the reference's W8A8 torch-op linears and SDPA attention).
* Two gloo ranks: the Ulysses split (text/image rows per rank, qkv rows permuted to the
  per-rank send layout, all-to-all of q/k/v and of the attention output, segmented quantizer
  reads) gives bit for bit the one-rank result.
"""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from diffucore_b200 import flux
from tests.conftest import GOLDEN, bits_to_torch
from tests.flux_torch_ops import TorchOps

CFG = dict(in_channels=64, context_in_dim=64, vec_in_dim=32, hidden_size=256, mlp_ratio=4.0, num_heads=2,
           depth=2, depth_single_blocks=2, axes_dim=(16, 56, 56), theta=10_000, qkv_bias=True, guidance_embed=False)


def _fixture():
    with np.load(GOLDEN / "flux_tiny.npz") as z:
        return {k: z[k] for k in z.files}


def _model(group: int) -> flux.Flux:
    model = flux.Flux(flux.FluxConfig(**CFG))
    flux.init_random_(model, seed=0, device="cpu")
    flux.quantize_linears(model, model.block_linear_names(), "cpu", group=group)
    return model.eval()


def _inputs(fx):
    img = bits_to_torch(fx["img"], torch.bfloat16)[0]
    txt = bits_to_torch(fx["txt"], torch.bfloat16)[0]
    y = bits_to_torch(fx["y"], torch.bfloat16)
    return img, txt, y, torch.from_numpy(fx["img_ids"]), torch.from_numpy(fx["txt_ids"])


def _run(model, img, txt, y, iid, tid, times, pg=None, ops=None, overlap=False):
    runner = flux.FluxRunner(model, txt.shape[0], img.shape[0], process_group=pg, device="cpu",
                             ops=ops if ops is not None else TorchOps(), overlap_exchange=overlap)
    assert runner.overlap_exchange == (overlap and pg is not None)
    runner.set_positions(iid, tid)
    t0, t1 = runner.img_rows
    r0 = runner.rows[0]
    txt_loc = txt[r0: r0 + runner.t_loc]
    outs = []
    for t in times:
        ts = torch.full((1,), float(t), dtype=torch.bfloat16)
        outs.append(runner.forward(img[t0:t1], txt_loc, ts, y))
    return outs, (t0, t1)


@pytest.mark.parametrize("group", [0, 256])
def test_runner_reproduces_reference_flux(group):
    fx = _fixture()
    assert sorted(fx[f"names_g{group}"]) == sorted(_model(group).block_linear_names())
    img, txt, y, iid, tid = _inputs(fx)
    outs, _ = _run(_model(group), img, txt, y, iid, tid, fx["times"])
    for i, got in enumerate(outs):
        want = bits_to_torch(fx[f"v_g{group}_t{i}"], torch.bfloat16).float()
        assert got.shape == want.shape
        assert torch.isfinite(got).all()
        # every step rounds where the reference's torch ops round: the velocity is bit-identical
        assert torch.equal(got.float(), want), (got.float() - want).abs().max().item()


@pytest.mark.parametrize("group", [0, 256])
def test_cpu_baseline_ops_reproduce_reference_flux(group):
    """The ops bench.py times as the FLUX CPU baseline (oracle/torch_ref.py FluxOps: torch._int_mm
    for the int32 products, as the reference's torch-op path) give the reference's own velocity
    bit for bit, so that baseline runs the reference's arithmetic."""
    from oracle.torch_ref import FluxOps
    fx = _fixture()
    img, txt, y, iid, tid = _inputs(fx)
    outs, _ = _run(_model(group), img, txt, y, iid, tid, fx["times"], ops=FluxOps())
    for i, got in enumerate(outs):
        want = bits_to_torch(fx[f"v_g{group}_t{i}"], torch.bfloat16).float()
        assert torch.equal(got.float(), want), (got.float() - want).abs().max().item()


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _ulysses_worker(rank: int, world: int, port: int, group: int, path: str, overlap: bool = False) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        torch.manual_seed(0)
        fx = _fixture()
        img, txt, y, iid, tid = _inputs(fx)
        outs, (t0, t1) = _run(_model(group), img, txt, y, iid, tid, fx["times"], pg=dist.group.WORLD,
                              overlap=overlap)
        torch.save({"outs": outs, "rows": (t0, t1)}, f"{path}.{rank}")
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("group,overlap", [(0, False), (256, False), (256, True)])
def test_ulysses_two_ranks_match_one_rank(tmp_path, group, overlap):
    """Also with the single-stream blocks' q/k/v exchange started before their MLP GEMM
    (overlap_exchange): the asynchronous collective changes the schedule, not a bit."""
    fx = _fixture()
    img, txt, y, iid, tid = _inputs(fx)
    single, _ = _run(_model(group), img, txt, y, iid, tid, fx["times"])
    path = str(tmp_path / "out")
    mp.start_processes(_ulysses_worker, args=(2, _free_port(), group, path, overlap), nprocs=2, join=True,
                       start_method="spawn")
    parts = [torch.load(f"{path}.{r}") for r in range(2)]
    # rank 0 owns 68 rows: the 40 text tokens and image tokens 0..27; rank 1 image tokens 28..95
    assert parts[0]["rows"] == (0, 28) and parts[1]["rows"] == (28, 96)
    for i in range(len(single)):
        joined = torch.cat([parts[0]["outs"][i], parts[1]["outs"][i]], dim=0)
        assert torch.equal(joined, single[i])


WIDE = dict(CFG, hidden_size=1024, num_heads=8, depth=1, depth_single_blocks=1)


def _wide_model(group: int) -> flux.Flux:
    model = flux.Flux(flux.FluxConfig(**WIDE))
    flux.init_random_(model, seed=1, device="cpu")
    flux.quantize_linears(model, model.block_linear_names(), "cpu", group=group)
    return model.eval()


def _wide_inputs():
    g = torch.Generator().manual_seed(13)
    img = torch.randn(88, 64, generator=g).to(torch.bfloat16)            # 8 x 11 patches
    txt = torch.randn(40, 64, generator=g).to(torch.bfloat16)
    y = torch.randn(1, 32, generator=g).to(torch.bfloat16)
    return img, txt, y, flux.img_ids(16, 22, 2), flux.txt_ids(40)


def _wide_worker(rank: int, world: int, port: int, path: str) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        img, txt, y, iid, tid = _wide_inputs()
        outs, rows = _run(_wide_model(256), img, txt, y, iid, tid, (0.8,), pg=dist.group.WORLD)
        torch.save({"outs": outs, "rows": rows}, f"{path}.{rank}")
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [4, 8])
def test_ulysses_four_and_eight_ranks_match_one_rank(tmp_path, world):
    """8 heads, 40 text + 88 image tokens split over 4 and 8 gloo ranks (16 rows each at 8 ranks,
    so three ranks hold text rows and one holds both kinds): same velocity as one rank, bit for bit."""
    img, txt, y, iid, tid = _wide_inputs()
    single, _ = _run(_wide_model(256), img, txt, y, iid, tid, (0.8,))
    path = str(tmp_path / "out")
    mp.start_processes(_wide_worker, args=(world, _free_port(), path), nprocs=world, join=True,
                       start_method="spawn")
    parts = [torch.load(f"{path}.{r}") for r in range(world)]
    assert parts[0]["rows"][0] == 0 and parts[-1]["rows"][1] == 88
    joined = torch.cat([p["outs"][0] for p in parts], dim=0)
    assert torch.equal(joined, single[0])

