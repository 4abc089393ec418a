"""Parity at the headline size: bench.py's config-2 workload (B=4, H=32, S=8192,
D=128, bf16, block 128, every causal block kept with p=0.25, diagonal always,
bitmap seed 0) through the public backend, checked against the CPU oracle.

* CSR: the device compiler's block_pairs / block_pair_offsets equal the oracle's
  restatement of build_block_pairs_from_mask (patterns/base.py:36-89), bit-exact.
* Output: four (b, h) slices spread over the batch and heads against the fp32
  masked-dense oracle (masked_sdpa.py:23-68, chunked by query rows), within
  max-abs 2e-2 and mean-abs 2e-3; every slice finite.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
import sparseattentioninfer_b200 as sa
from oracle import patterns as op
from sparseattentioninfer_b200 import _capi, workloads as wl

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
B, H, S, D, BS, P_KEEP = 4, 32, 8192, 128, 128, 0.25
SLICES = ((0, 0), (1, 7), (2, 19), (3, 31))


def test_config2_full_size_csr_and_sampled_slices():
    bitmap = wl.bernoulli_block_bitmap(H, S // BS, S // BS, P_KEEP, seed=0)
    q, k, v = wl.seeded_qkv(1000, B, H, H, S, S, D, device=DEV, dtype=torch.bfloat16)
    md = sa.BlockMaskPattern(bitmap.to(DEV), BS).build(q, k)
    rp, ro = op.csr_from_block_bitmap(bitmap.numpy())
    assert np.array_equal(md.block_pair_offsets.cpu().numpy(), ro)
    got_pairs = md.block_pairs.cpu().numpy()
    for h in range(H):
        n = ro[h, -1]
        assert np.array_equal(got_pairs[h, :n], rp[h, :n]), h
    out = sa.get_backend("cuda_sm100").forward(q, k, v, md)
    assert _capi.device_error() == 0
    assert bool(torch.isfinite(out).all())
    for b, h in SLICES:
        qs, ks, vs = (t[b:b + 1, h:h + 1].float().cpu() for t in (q, k, v))
        bm = bitmap[h].bool()
        keep = (lambda _h, r0, r1, bm=bm: bm[torch.arange(r0, r1) // BS][:, torch.arange(S) // BS])
        ref = oracle.masked_sdpa_chunked(qs, ks, vs, keep, row_chunk=1024)
        err = (out[b:b + 1, h:h + 1].float().cpu() - ref).abs()
        assert err.max().item() <= 2e-2 and err.mean().item() <= 2e-3, (b, h, err.max().item(), err.mean().item())
