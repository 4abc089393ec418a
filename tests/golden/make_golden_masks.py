"""Golden token masks from the REFERENCE's own pattern classes (their
``_get_mask``: BigBirdPattern bigbird_pattern.py:173-210, BigBirdKeepRatioPattern
:487-531, BigBird2Pattern :648-), for the device-built ``materialize_mask=True``
masks of this package to be compared with bit for bit.

Run in the build container (where the reference checkout is importable):

    python tests/golden/make_golden_masks.py --reference <path-to-SparseAttentionInfer>

Writes ``masks.npz`` (each mask [H, T_q, T_k] bool, np.packbits along T_k) and
``masks_manifest.json`` (how each was built).
"""
from __future__ import annotations

import argparse
import json
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    args = ap.parse_args()
    sys.path.insert(0, args.reference)
    from sparse_attentions.patterns import BigBird2Pattern, BigBirdKeepRatioPattern, BigBirdPattern

    def dummy(H, T):
        return torch.zeros(1, H, T, 8)

    out: dict[str, np.ndarray] = {}
    manifest: dict = {}

    def put(name, pat, H, T_q, T_k, meta):
        md = pat.build(dummy(H, T_q), dummy(H, T_k))
        m = md.mask.numpy().astype(np.uint8)
        out[name] = np.packbits(m, axis=-1)
        manifest[name] = dict(meta, H=H, T_q=T_q, T_k=T_k, block_size=md.block_size)

    def injected(layouts, H, n_kv=None):
        pat = BigBirdKeepRatioPattern(keep_ratio=0.5, n_heads=H) if n_kv is None else \
            BigBirdKeepRatioPattern(group_sparsities=[0.5] * n_kv, n_heads=H, n_kv_heads=n_kv)
        return pat

    for name, layouts, H, n_kv, T_q, T_k in [
        ("keep_cfg1_prefill", [(64, 2, 3, 2)], 8, None, 1024, 1024),
        ("keep_cfg4_decode", [(64, 2, 4, 2)], 8, None, 1, 1000),
        ("keep_chunked", [(64, 2, 3, 2)], 4, None, 256, 1000),
        ("keep_groups", [(64, 1, 2, 3), (64, 3, 5, 1)], 8, 2, 512, 512),
    ]:
        pat = injected(layouts, H, n_kv)
        pat._layout_cache[(T_q, T_k)] = tuple(tuple(x) for x in layouts)
        put(name, pat, H, T_q, T_k, dict(kind="layouts", layouts=[list(x) for x in layouts], n_kv_heads=n_kv))
    for name, top_k, H, T_q, T_k in [("bigbird_topk256_prefill", 256, 8, 1024, 1024),
                                     ("bigbird_topk256_decode", 256, 8, 1, 1000)]:
        put(name, BigBirdPattern(top_k=top_k, n_heads=H), H, T_q, T_k, dict(kind="bigbird_topk", top_k=top_k))
    put("bigbird2_topk256_prefill", BigBird2Pattern(top_k=256, n_heads=4), 4, 1024, 1024,
        dict(kind="bigbird2_topk", top_k=256))

    np.savez_compressed(HERE / "masks.npz", **out)
    (HERE / "masks_manifest.json").write_text(json.dumps(manifest, indent=1, sort_keys=True))


if __name__ == "__main__":
    main()
