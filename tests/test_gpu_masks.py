"""Token masks built on the device (``materialize_mask=True``) against the
reference's own ``_get_mask`` outputs (tests/golden/make_golden_masks.py):
BigBirdPattern (bigbird_pattern.py:173-210), BigBirdKeepRatioPattern (:487-531,
including per-KV-group layouts and a chunk whose T_k - T_q is not a multiple of
the block) and BigBird2Pattern (:648-). Bit-exact: block mask, causal rule and
the forced diagonal (:527-529)."""
from __future__ import annotations

import json

import numpy as np
import pytest
import torch

import sparseattentioninfer_b200 as sa
from tests.conftest import GOLDEN

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
MAN = json.loads((GOLDEN / "masks_manifest.json").read_text())


def _pattern(meta):
    if meta["kind"] == "layouts":
        return sa.BigBirdKeepRatioPattern(layouts=meta["layouts"], n_heads=meta["H"], materialize_mask=True)
    if meta["kind"] == "bigbird_topk":
        return sa.BigBirdPattern(top_k=meta["top_k"], n_heads=meta["H"], materialize_mask=True)
    return sa.BigBird2Pattern(top_k=meta["top_k"], n_heads=meta["H"], materialize_mask=True)


@pytest.mark.parametrize("name", sorted(MAN))
def test_device_mask_equals_reference_get_mask(name):
    meta = MAN[name]
    H, T_q, T_k = meta["H"], meta["T_q"], meta["T_k"]
    with np.load(GOLDEN / "masks.npz") as z:
        ref = np.unpackbits(z[name], axis=-1, count=T_k).astype(bool)
    q = torch.zeros(1, H, T_q, 64, device=DEV, dtype=torch.bfloat16)
    k = torch.zeros(1, H, T_k, 64, device=DEV, dtype=torch.bfloat16)
    md = _pattern(meta).build(q, k)
    assert md.block_size == meta["block_size"]
    got = md.mask.cpu().numpy().astype(bool)
    assert got.shape == ref.shape
    diff = np.argwhere(got != ref)
    assert diff.size == 0, f"{name}: {len(diff)} entries differ, first {diff[:3].tolist()}"
