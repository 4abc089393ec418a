"""Tensor-parallel Qwen3 host logic on CPU: KV-group sharding, weight slicing and
the two all-reduces per layer, on gloo ranks (world size 2) with the oracle's
checker kernels standing in for the CUDA attention calls."""
from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from oracle.qwen3_model import CheckerKernels, masked_dense_forward
from sparseattentioninfer_b200 import tp

ARCH = tp.Qwen3Arch(hidden=128, layers=2, heads=8, kv_heads=4, head_dim=32, intermediate=256, vocab=300)
LAYOUT = (32, 1, 2, 2)
T, STEPS = 256, 3


def test_kv_group_shard_partitions():
    for world in (1, 2, 4, 8):
        spans = [tp.kv_group_shard(8, r, world) for r in range(world)]
        assert spans[0][0] == 0 and spans[-1][1] == 8
        assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
    with pytest.raises(ValueError):
        tp.kv_group_shard(8, 0, 3)
    with pytest.raises(ValueError):
        tp.kv_group_shard(8, 2, 2)
    with pytest.raises(ValueError):
        tp.even_shard(12288, 0, 5)


def test_weight_shards_reassemble():
    full = tp.Qwen3TPWeights(ARCH, 0, 1, seed=5, device="cpu", dtype=torch.float32)
    parts = [tp.Qwen3TPWeights(ARCH, r, 2, seed=5, device="cpu", dtype=torch.float32) for r in range(2)]
    D, H, Hkv = ARCH.head_dim, ARCH.heads, ARCH.kv_heads
    for li in range(ARCH.layers):
        F, P = full.layers[li], [p.layers[li] for p in parts]
        q = torch.cat([p["qkv"][: p_.hq * D] for p, p_ in zip(P, parts)], 0)
        assert torch.equal(q, F["qkv"][: H * D])
        assert torch.equal(torch.cat([p["o"] for p in P], 1), F["o"])
        assert torch.equal(torch.cat([p["down"] for p in P], 1), F["down"])
        inter = ARCH.intermediate
        g = torch.cat([p["gu"][: inter // 2] for p in P], 0)
        assert torch.equal(g, F["gu"][:inter])
    assert parts[1].q_lo == H // 2 and parts[1].kv_lo == Hkv // 2


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank: int, world: int, port: int, out_path: str):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.distributed.init_process_group("gloo", rank=rank, world_size=world)
    try:
        torch.manual_seed(0)
        w = tp.Qwen3TPWeights(ARCH, rank, world, seed=11, device="cpu", dtype=torch.float32)
        r = tp.Qwen3TPRunner(w, 2, T + STEPS, LAYOUT, sparse_layers=[0], kernels=CheckerKernels)
        tok = torch.randint(0, ARCH.vocab, (2, T), generator=torch.Generator().manual_seed(1))
        logits = [r.prefill(tok, chunk=64)]
        t = logits[0].argmax(-1, keepdim=True)
        toks = [t]
        for _ in range(STEPS):
            t, lg = r.step(t, return_logits=True)
            logits.append(lg)
            toks.append(t)
        if rank == 0:
            torch.save({"logits": logits, "toks": toks, "tok": tok}, out_path)
    finally:
        torch.distributed.destroy_process_group()


def test_tp2_gloo_matches_masked_dense_oracle(tmp_path):
    out = str(tmp_path / "tp2.pt")
    mp.start_processes(_rank_main, args=(2, _free_port(), out), nprocs=2, join=True, start_method="spawn")
    res = torch.load(out)
    full = tp.Qwen3TPWeights(ARCH, 0, 1, seed=11, device="cpu", dtype=torch.float32)
    cache = []
    ref = [masked_dense_forward(full, res["tok"], LAYOUT, [0], cache)]
    for t in res["toks"][:-1]:
        ref.append(masked_dense_forward(full, t, LAYOUT, [0], cache))
    for a, b in zip(res["logits"], ref):
        assert (a - b).abs().max().item() < 1e-4
