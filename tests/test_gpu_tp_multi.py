"""Tensor-parallel runner on 2 GPUs (NCCL, one process per GPU): prefill, eager
decode and graph-replayed decode give the single-GPU run's logits (the
all-reduce changes only the summation order: max-abs <= 2e-2 * max|logit|).
Skipped when fewer than 2 GPUs are visible."""
from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from sparseattentioninfer_b200 import tp

pytestmark = pytest.mark.gpu
ARCH = tp.Qwen3Arch(hidden=512, layers=2, heads=32, kv_heads=8, head_dim=128, intermediate=1024, vocab=2000)
LAYOUT, T, STEPS = (128, 2, 4, 3), 1280, 6


def _run(rank: int, world: int, out_path: str | None):
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    w = tp.Qwen3TPWeights(ARCH, rank, world, seed=21, device=dev)
    r = tp.Qwen3TPRunner(w, 2, T + 2 * STEPS, LAYOUT)
    tok = torch.randint(0, ARCH.vocab, (2, T), generator=torch.Generator().manual_seed(8)).to(dev)
    logits = [r.prefill(tok, chunk=512).cpu()]
    t = logits[0].argmax(-1, keepdim=True).to(dev)
    for _ in range(STEPS):
        t, lg = r.step(t, return_logits=True)
        logits.append(lg.cpu())
    r.capture_decode()
    g = r.step_graph(t)
    for i in range(STEPS):
        logits.append(r.graph_logits.cpu())
        if i + 1 < STEPS:
            g = r.step_graph()
    torch.cuda.synchronize()
    if out_path is not None and rank == 0:
        torch.save(logits, out_path)
    return logits


def _rank_main(rank: int, world: int, port: int, out_path: str):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.distributed.init_process_group("nccl", rank=rank, world_size=world,
                                         device_id=torch.device("cuda", rank))
    try:
        _run(rank, world, out_path)
    finally:
        torch.distributed.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_tp2_nccl_matches_single_gpu(tmp_path):
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    out = str(tmp_path / "tp2.pt")
    mp.start_processes(_rank_main, args=(2, port, out), nprocs=2, join=True, start_method="spawn")
    got = torch.load(out)
    ref = _run(0, 1, None)
    assert len(got) == len(ref)
    for i, (a, b) in enumerate(zip(got, ref)):
        scale = b.abs().max().item()
        assert (a - b).abs().max().item() <= 2e-2 * scale, f"position {i}"
