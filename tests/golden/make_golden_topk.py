"""Golden fixtures for the data-dependent top-k pattern, produced by the
REFERENCE's own code: TopKPattern.build (sparse_attentions/patterns/
topk_pattern.py:44-62) and MaskedSdpaBackend.forward with kind "topk"
(sparse_attentions/attention/masked_sdpa.py:51-63).

    python tests/golden/make_golden_topk.py --reference <path-to-SparseAttentionInfer>

Writes ``topk_cases.npz`` (fp32 outputs, keep ratios) and ``topk_manifest.json``
(seeds and shapes). Inputs are tests.golden.make_golden.seeded_qkv draws; GQA
K/V are repeated per query head (repeat_kv) before the reference runs, as its
Qwen3 hook does.
"""
from __future__ import annotations

import argparse
import json
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
from make_golden import seeded_qkv  # noqa: E402

# name: (seed, B, H, Hkv, T_q, T_k, D, dtype, top_k)
CASES = {
    "topk_prefill_fp32": (21, 1, 4, 4, 256, 256, 64, "fp32", 32),
    "topk_prefill_gqa_bf16": (22, 1, 8, 2, 256, 256, 128, "bf16", 48),
    "topk_decode_gqa_bf16": (23, 3, 8, 2, 1, 1000, 128, "bf16", 64),
    "topk_k_exceeds_rows": (24, 1, 2, 2, 64, 64, 64, "fp32", 100),
}


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    args = ap.parse_args()
    sys.path.insert(0, args.reference)
    from sparse_attentions.attention.masked_sdpa import MaskedSdpaBackend
    from sparse_attentions.patterns.topk_pattern import TopKPattern

    backend = MaskedSdpaBackend()
    out: dict[str, np.ndarray] = {}
    manifest: dict = {}
    for name, (seed, B, H, Hkv, T_q, T_k, D, dtype, top_k) in CASES.items():
        q, k, v = seeded_qkv(seed, B, H, Hkv, T_q, T_k, D, dtype)
        kr, vr = k.repeat_interleave(H // Hkv, 1), v.repeat_interleave(H // Hkv, 1)
        md = TopKPattern(top_k).build(q, kr)
        out[name] = backend.forward(q, kr, vr, md).numpy().astype(np.float32)
        manifest[name] = dict(seed=seed, B=B, H=H, Hkv=Hkv, T_q=T_q, T_k=T_k, D=D, dtype=dtype, top_k=top_k,
                              keep_ratio=float(md.keep_ratio))
    np.savez_compressed(HERE / "topk_cases.npz", **out)
    (HERE / "topk_manifest.json").write_text(json.dumps(manifest, indent=1))


if __name__ == "__main__":
    main()
