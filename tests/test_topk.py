"""Data-dependent top-k attention (TopKPattern) against fixtures made by the
reference's own TopKPattern + MaskedSdpaBackend (tests/golden/make_golden_topk.py):
the oracle restatement on CPU, the CUDA path through the backend on the GPU
(bf16 outputs within max-abs 2e-2 / mean-abs 2e-3 of the fp32 reference)."""
from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import pytest
import torch

import oracle
import sparseattentioninfer_b200 as sa
from tests._inputs import seeded_qkv

GOLDEN = Path(__file__).resolve().parent / "golden"
MANIFEST = json.loads((GOLDEN / "topk_manifest.json").read_text())
with np.load(GOLDEN / "topk_cases.npz") as _z:
    CASES = {k: _z[k] for k in _z.files}
DEV = "cuda:0"


def _inputs(meta):
    return seeded_qkv(meta["seed"], meta["B"], meta["H"], meta["Hkv"], meta["T_q"], meta["T_k"], meta["D"],
                      meta["dtype"])


@pytest.mark.parametrize("name", sorted(MANIFEST))
def test_oracle_topk_matches_reference_fixture(name):
    meta = MANIFEST[name]
    q, k, v = _inputs(meta)
    rep = meta["H"] // meta["Hkv"]
    out = oracle.topk_sdpa(q, k.repeat_interleave(rep, 1), v.repeat_interleave(rep, 1), meta["top_k"])
    np.testing.assert_allclose(out.numpy(), CASES[name], atol=2e-5, rtol=0)


@pytest.mark.parametrize("name", sorted(MANIFEST))
def test_topk_pattern_keep_ratio(name):
    meta = MANIFEST[name]
    q = torch.zeros(1, meta["H"], meta["T_q"], 8)
    k = torch.zeros(1, meta["H"], meta["T_k"], 8)
    md = sa.TopKPattern(meta["top_k"]).build(q, k)
    assert md.kind == "topk" and md.topk == meta["top_k"]
    assert md.keep_ratio == pytest.approx(meta["keep_ratio"], abs=1e-12)


def _close(out, ref, what):
    o = out.float().cpu().numpy()
    err = np.abs(o - ref)
    assert np.isfinite(o).all(), what
    assert err.max() <= 2e-2 and err.mean() <= 2e-3, f"{what}: max {err.max():.3e} mean {err.mean():.3e}"


@pytest.mark.gpu
@pytest.mark.parametrize("name", sorted(MANIFEST))
def test_cuda_topk_matches_reference_fixture(name):
    meta = MANIFEST[name]
    q, k, v = _inputs(meta)
    dt = torch.float32 if meta["dtype"] == "fp32" else torch.bfloat16
    q, k, v = (t.to(DEV, dt) for t in (q, k, v))
    be = sa.get_backend("cuda_sm100")
    out = be.forward(q, k, v, sa.TopKPattern(meta["top_k"]).build(q, k))
    assert out.dtype == dt and be.actual_backend == "cuda_sm100"
    _close(out, CASES[name], name)


@pytest.mark.gpu
def test_cuda_topk_chunked_rows_and_larger_shape():
    """Several score chunks (small max_score_bytes) and a longer GQA prefill against
    the oracle; two calls give the same output."""
    from sparseattentioninfer_b200 import ops
    q, k, v = seeded_qkv(31, 1, 8, 2, 1536, 1536, 128, "bf16")
    ref = oracle.topk_sdpa(q, k.repeat_interleave(4, 1), v.repeat_interleave(4, 1), 96).numpy()
    qd, kd, vd = (t.to(DEV, torch.bfloat16) for t in (q, k, v))
    a = ops.topk_attention(qd, kd, vd, 96, max_score_bytes=4 << 20)
    b = ops.topk_attention(qd, kd, vd, 96)
    _close(a, ref, "chunked")
    assert torch.equal(a, b)
