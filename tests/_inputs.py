"""Seeded inputs of the golden cases (same draws as tests/golden/make_golden.py)."""
from __future__ import annotations

import numpy as np
import torch


def seeded_qkv(seed, B, H, Hkv, T_q, T_k, D, dtype):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, H, T_q, D, generator=g)
    k = torch.randn(B, Hkv, T_k, D, generator=g)
    v = torch.randn(B, Hkv, T_k, D, generator=g)
    if dtype == "bf16":
        q, k, v = (t.to(torch.bfloat16).float() for t in (q, k, v))
    return q, k, v


def case_inputs(meta):
    q, k, v = seeded_qkv(meta["seed"], meta["B"], meta["H"], meta["Hkv"], meta["T_q"], meta["T_k"], meta["D"],
                         meta["dtype"])
    sums = [float(t.double().sum()) for t in (q, k, v)]
    assert np.allclose(sums, meta["checksum"], rtol=0, atol=1e-6), "input generator drifted from the fixtures"
    return q, k, v


def expand_bitmap(bm, bs, T_q, T_k):
    t = torch.from_numpy(np.asarray(bm).astype(bool))
    q2b = torch.arange(T_q) // bs
    k2b = torch.arange(T_k) // bs
    return t[:, q2b][:, :, k2b]


def layouts_of(meta):
    return [tuple(x) for x in meta["layouts"]]
