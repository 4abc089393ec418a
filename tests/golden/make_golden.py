"""Generate the golden fixtures by running the REFERENCE's own Python code.

Run in the build container (where the reference checkout is importable):

    python tests/golden/make_golden.py --reference <path-to-SparseAttentionInfer>

It imports the reference's pattern classes (sparse_attentions/patterns/*.py),
build_block_pairs_from_mask / kv_block_list_to_pairs (patterns/base.py) and
MaskedSdpaBackend (attention/masked_sdpa.py), and writes what they return:

* ``csr_cases.npz``  — block_pairs / block_pair_offsets (+ kv_block_list,
  keep_ratio) of BigBird, BigBird-keep-ratio (single and per-KV-group),
  injected BASELINE layouts, BigBird2, LocalWindow, arbitrary token masks and
  padded lists, for prefill and decode shapes;
* ``attn_<name>.npz`` — fp32 MaskedSdpaBackend outputs on seeded inputs.

Inputs are regenerated in the tests from the seeds recorded here
(torch.Generator().manual_seed(seed), draw order q, k, v); the manifest keeps
a checksum of each input so a drift in the generator is caught. Inputs of the
bf16 cases are rounded to bf16 before the fp32 reference runs, so the CUDA
kernel sees exactly the values the reference saw.
"""
from __future__ import annotations

import argparse
import json
import math
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent


def seeded_qkv(seed: int, B: int, H: int, Hkv: int, T_q: int, T_k: int, D: int, dtype: str):
    """Shared with the tests: N(0,1) draws in the order q, k, v from one generator."""
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, H, T_q, D, generator=g)
    k = torch.randn(B, Hkv, T_k, D, generator=g)
    v = torch.randn(B, Hkv, T_k, D, generator=g)
    if dtype == "bf16":
        q, k, v = (t.to(torch.bfloat16).float() for t in (q, k, v))
    return q, k, v


def generator_bigbird_bitmap(H: int, nb: int, window: int, n_global: int, n_random: int, seed: int) -> np.ndarray:
    """Block bitmap of the CPU-runnable BigBird layer as the task statement
    words it (random blocks from torch.Generator seed 1), which no reference
    pattern class implements (the reference rotates deterministically).
    Per head h, per query block qb in order: window [qb-window+1, qb], global
    blocks [0, n_global) (global rows see every earlier block, which for rows
    < n_global is already the window/causal set), then n_random blocks drawn
    with torch.randperm over the remaining earlier blocks in ascending order."""
    g = torch.Generator().manual_seed(seed)
    bm = np.zeros((H, nb, nb), dtype=np.uint8)
    for h in range(H):
        for qb in range(nb):
            keep = set(range(max(0, qb - window + 1), qb + 1))
            keep |= set(range(min(n_global, qb + 1)))
            if qb < n_global:
                keep |= set(range(qb + 1))
            cands = [b for b in range(qb) if b not in keep]
            if cands:
                perm = torch.randperm(len(cands), generator=g)[: n_random].tolist()
                keep |= {cands[i] for i in perm}
            for kb in keep:
                bm[h, qb, kb] = 1
    return bm


def expand_bitmap(bm: np.ndarray, bs: int, T_q: int, T_k: int) -> torch.Tensor:
    t = torch.from_numpy(bm.astype(bool))
    q2b = torch.arange(T_q) // bs
    k2b = torch.arange(T_k) // bs
    return t[:, q2b][:, :, k2b]


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    args = ap.parse_args()
    sys.path.insert(0, args.reference)
    from sparse_attentions.attention.masked_sdpa import MaskedSdpaBackend
    from sparse_attentions.patterns import (
        BigBird2Pattern,
        BigBirdKeepRatioPattern,
        BigBirdPattern,
        LocalWindowPattern,
    )
    from sparse_attentions.patterns.base import (
        PatternMetadata,
        build_block_pairs_from_mask,
        kv_block_list_to_pairs,
    )

    manifest: dict = {"csr": {}, "attn": {}}
    csr: dict[str, np.ndarray] = {}

    def dummy(H, T):
        return torch.zeros(1, H, T, 8)

    def put_pattern(name, pat, H, T_q, T_k, meta: dict):
        md = pat.build(dummy(H, T_q), dummy(H, T_k))
        csr[f"{name}.pairs"] = md.block_pairs.numpy().astype(np.int32)
        csr[f"{name}.offsets"] = md.block_pair_offsets.numpy().astype(np.int32)
        if md.kv_block_list is not None:
            csr[f"{name}.kvl"] = md.kv_block_list.numpy().astype(np.int32)
        manifest["csr"][name] = dict(meta, H=H, T_q=T_q, T_k=T_k, block_size=md.block_size,
                                     keep_ratio=md.keep_ratio)
        return md

    # --- BigBirdPattern (top_k driven layout; rotation per q-head) -------------
    for top_k, H, T_q, T_k in [(64, 4, 512, 512), (256, 8, 1024, 1024), (256, 8, 1, 1000), (1024, 4, 2048, 2048)]:
        put_pattern(f"bigbird_topk{top_k}_H{H}_q{T_q}_k{T_k}", BigBirdPattern(top_k=top_k, n_heads=H), H, T_q, T_k,
                    dict(kind="bigbird_topk", top_k=top_k))
    # --- BigBird2Pattern ------------------------------------------------------
    for top_k, H, T_q, T_k in [(256, 4, 1024, 1024), (256, 4, 1, 777)]:
        put_pattern(f"bigbird2_topk{top_k}_H{H}_q{T_q}_k{T_k}", BigBird2Pattern(top_k=top_k, n_heads=H), H, T_q, T_k,
                    dict(kind="bigbird2_topk", top_k=top_k))
    # --- BigBirdKeepRatioPattern: single ratio and per-KV-group sparsities ----
    for kr, H, T_q, T_k in [(0.3, 8, 1024, 1024), (0.3, 8, 1, 1000), (0.05, 4, 4096, 4096)]:
        put_pattern(f"keep{kr}_H{H}_q{T_q}_k{T_k}", BigBirdKeepRatioPattern(keep_ratio=kr, n_heads=H), H, T_q, T_k,
                    dict(kind="keep_ratio", keep_ratio_in=kr))
    gs = [0.5, 0.8, 0.2, 0.9]
    for T_q, T_k in [(2048, 2048), (1, 2047)]:
        put_pattern(f"groups_H16_q{T_q}_k{T_k}",
                    BigBirdKeepRatioPattern(group_sparsities=gs, n_heads=16, n_kv_heads=4), 16, T_q, T_k,
                    dict(kind="group_sparsities", group_sparsities=gs, n_kv_heads=4))

    # --- injected BASELINE layouts (layout cache of BigBirdKeepRatioPattern) ---
    def injected(name, layouts, H, T_q, T_k, n_kv=None):
        pat = BigBirdKeepRatioPattern(keep_ratio=0.5, n_heads=H) if len(layouts) == 1 else \
            BigBirdKeepRatioPattern(group_sparsities=[0.5] * len(layouts), n_heads=H, n_kv_heads=len(layouts))
        pat._layout_cache[(T_q, T_k)] = tuple(tuple(x) for x in layouts)
        return put_pattern(name, pat, H, T_q, T_k, dict(kind="layouts", layouts=[list(x) for x in layouts]))

    c1 = injected("cfg1_layout", [(64, 2, 3, 2)], 8, 1024, 1024)
    rng = np.random.default_rng(2)
    cfg3_layouts = [(64, int(rng.integers(1, 5)), int(rng.integers(2, 9)), int(rng.integers(0, 4))) for _ in range(8)]
    injected("cfg3_small", cfg3_layouts, 32, 2048, 2048)
    injected("cfg4_decode", [(64, 2, 4, 2)], 32, 1, 32768 + 37)
    injected("cfg4_decode_short", [(64, 2, 4, 2)], 32, 1, 100)
    injected("cfg5_layout", [(128, 2, 4, 3)], 8, 4096, 4096)
    injected("chunked_prefill", [(64, 2, 3, 2)], 4, 256, 1024)

    # --- LocalWindowPattern (token mask -> build_block_pairs_from_mask) -------
    for W, bs, T in [(100, 32, 512), (64, 64, 300)]:
        md = LocalWindowPattern(window_size=W, block_size=bs).build(dummy(2, T), dummy(2, T))
        name = f"local_w{W}_bs{bs}_T{T}"
        csr[f"{name}.pairs"] = md.block_pairs.numpy().astype(np.int32)
        csr[f"{name}.offsets"] = md.block_pair_offsets.numpy().astype(np.int32)
        manifest["csr"][name] = dict(kind="local", window=W, H=2, T_q=T, T_k=T, block_size=bs)

    # --- arbitrary token masks -> build_block_pairs_from_mask -----------------
    g = torch.Generator().manual_seed(7)
    for H, T_q, T_k, bs, dens in [(3, 300, 300, 32, 0.002), (2, 1, 500, 64, 0.05), (2, 256, 256, 16, 0.0)]:
        m = torch.rand(H, T_q, T_k, generator=g) < dens
        if dens == 0.0:
            m[1, 5, 7] = True  # one head empty, one with a single kept token
        pairs, offs = build_block_pairs_from_mask(m, bs)
        name = f"tokmask_H{H}_q{T_q}_k{T_k}_bs{bs}"
        csr[f"{name}.mask"] = np.packbits(m.numpy().astype(np.uint8), axis=-1)
        csr[f"{name}.pairs"] = pairs.numpy().astype(np.int32)
        csr[f"{name}.offsets"] = offs.numpy().astype(np.int32)
        manifest["csr"][name] = dict(kind="token_mask", H=H, T_q=T_q, T_k=T_k, block_size=bs)

    # --- padded legacy list -> kv_block_list_to_pairs -------------------------
    kvl = torch.randint(-1, 40, (3, 9, 6), generator=g, dtype=torch.int32)
    pairs, offs = kv_block_list_to_pairs(kvl)
    csr["kvlist_random.kvl"] = kvl.numpy()
    csr["kvlist_random.pairs"] = pairs.numpy().astype(np.int32)
    csr["kvlist_random.offsets"] = offs.numpy().astype(np.int32)
    manifest["csr"]["kvlist_random"] = dict(kind="kvlist")

    np.savez_compressed(HERE / "csr_cases.npz", **csr)

    # --- attention outputs through MaskedSdpaBackend --------------------------
    backend = MaskedSdpaBackend()

    def run_attn(name, seed, B, H, Hkv, T_q, T_k, D, dtype, mask, meta):
        q, k, v = seeded_qkv(seed, B, H, Hkv, T_q, T_k, D, dtype)
        kr = k.repeat_interleave(H // Hkv, dim=1)  # repeat_kv, as the reference hook does
        vr = v.repeat_interleave(H // Hkv, dim=1)
        out = backend.forward(q, kr, vr, PatternMetadata(kind="mask", mask=mask))
        np.savez_compressed(HERE / f"attn_{name}.npz", out=out.numpy().astype(np.float32))
        manifest["attn"][name] = dict(meta, seed=seed, B=B, H=H, Hkv=Hkv, T_q=T_q, T_k=T_k, D=D, dtype=dtype,
                                      checksum=[float(q.double().sum()), float(k.double().sum()),
                                                float(v.double().sum())])

    # config 1 with the reference's own rotation layout (64, 2, 3, 2)
    run_attn("cfg1_rotation", 0, 1, 8, 8, 1024, 1024, 64, "fp32", c1.mask,
             dict(pattern="layouts", layouts=[[64, 2, 3, 2]], block_size=64))
    # config 1 as worded (Generator seed 1 random blocks): bitmap -> token mask ->
    # reference build_block_pairs_from_mask + MaskedSdpaBackend
    bm1 = generator_bigbird_bitmap(8, 16, 3, 2, 2, seed=1)
    m1 = expand_bitmap(bm1, 64, 1024, 1024)
    p1, o1 = build_block_pairs_from_mask(m1, 64)
    csr["cfg1_generator.bitmap"] = bm1
    csr["cfg1_generator.pairs"] = p1.numpy().astype(np.int32)
    csr["cfg1_generator.offsets"] = o1.numpy().astype(np.int32)
    manifest["csr"]["cfg1_generator"] = dict(kind="bitmap", H=8, T_q=1024, T_k=1024, block_size=64)
    run_attn("cfg1_generator", 0, 1, 8, 8, 1024, 1024, 64, "fp32", m1, dict(pattern="bitmap", block_size=64))
    np.savez_compressed(HERE / "csr_cases.npz", **csr)

    # arbitrary Bernoulli block mask (config-2 shape family, reduced S)
    gb = torch.Generator().manual_seed(11)
    nb = 8
    u = torch.rand(2, nb, nb, generator=gb)
    qb = torch.arange(nb).view(1, -1, 1)
    kb = torch.arange(nb).view(1, 1, -1)
    bm2 = (((u < 0.25) & (kb <= qb)) | (kb == qb)).numpy().astype(np.uint8)
    csr["bern_small.bitmap"] = bm2
    np.savez_compressed(HERE / "csr_cases.npz", **csr)
    run_attn("bern_small", 3, 1, 2, 2, 1024, 1024, 128, "bf16", expand_bitmap(bm2, 128, 1024, 1024),
             dict(pattern="bitmap", block_size=128, bitmap="bern_small"))

    # GQA with per-group layouts (config-3 family, reduced S)
    gqa_layouts = [(64, 1, 2, 3), (64, 3, 5, 1)]
    pat = BigBirdKeepRatioPattern(group_sparsities=[0.5, 0.5], n_heads=8, n_kv_heads=2)
    pat._layout_cache[(512, 512)] = tuple(gqa_layouts)
    md = pat.build(dummy(8, 512), dummy(8, 512))
    run_attn("gqa_groups", 4, 1, 8, 2, 512, 512, 128, "bf16", md.mask,
             dict(pattern="layouts", layouts=[list(x) for x in gqa_layouts], block_size=64))

    # decode (T_q = 1, T_k not a multiple of the block size), GQA
    pat = BigBirdKeepRatioPattern(keep_ratio=0.5, n_heads=8)
    pat._layout_cache[(1, 1000)] = ((64, 2, 4, 2),)
    md = pat.build(dummy(8, 1), dummy(8, 1000))
    run_attn("decode_gqa", 5, 2, 8, 2, 1, 1000, 128, "bf16", md.mask,
             dict(pattern="layouts", layouts=[[64, 2, 4, 2]], block_size=64))

    # prefill with T not a multiple of the block size, D = 64
    pat = BigBirdKeepRatioPattern(keep_ratio=0.5, n_heads=2)
    pat._layout_cache[(200, 200)] = ((64, 1, 2, 1),)
    md = pat.build(dummy(2, 200), dummy(2, 200))
    run_attn("ragged_d64", 6, 1, 2, 2, 200, 200, 64, "bf16", md.mask,
             dict(pattern="layouts", layouts=[[64, 1, 2, 1]], block_size=64))

    (HERE / "manifest.json").write_text(json.dumps(manifest, indent=1, sort_keys=True))
    print("wrote", sorted(p.name for p in HERE.glob("*.npz")))


if __name__ == "__main__":
    main()
