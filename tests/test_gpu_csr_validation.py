"""CSR validation (sa_validate_csr, ops.validate_csr, CudaSm100Backend.forward):
the properties the kernels rely on. The reference's builders emit sorted rows
starting at offset 0 (patterns/base.py:75-89, bigbird_pattern.py:533-583); a
caller CSR that breaks them is rejected with SA_ERR_CSR instead of being read."""
from __future__ import annotations

import re

import pytest
import torch

import sparseattentioninfer_b200 as sa
from sparseattentioninfer_b200 import _capi, ops, workloads
from sparseattentioninfer_b200.patterns import PatternMetadata

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
H, T, D, BS = 2, 512, 128, 128   # NQB = NKB = 4


def _good():
    pairs = torch.tensor([[0, 0, 1, 0, 2, 1, 3, 0, 0, 0], [0, 1, 1, 2, 3, 0, 0, 0, 0, 0]], dtype=torch.int32)
    offs = torch.tensor([[0, 1, 3, 5, 7], [0, 1, 2, 3, 5]], dtype=torch.int32)
    return pairs.to(DEV), offs.to(DEV)


def test_valid_csr_passes():
    pairs, offs = _good()
    ops.validate_csr(pairs, offs, T, T, BS)


@pytest.mark.parametrize("mutate,what", [
    (lambda p, o: p.__setitem__((0, 1), 1) or p.__setitem__((0, 2), 0), "strictly increasing"),   # unsorted row
    (lambda p, o: o.__setitem__((1, 2), 0), "decrease"),                                          # non-monotone
    (lambda p, o: p.__setitem__((1, 4), 9), "outside [0, NKB)"),                                  # out of range
    (lambda p, o: o.__setitem__((0, 0), 1), "!= 0"),                                              # offsets[h,0] != 0
    (lambda p, o: o.__setitem__((1, 4), 11), "pairs_stride"),                                     # past the width
])
def test_invalid_csr_is_rejected(mutate, what):
    pairs, offs = _good()
    mutate(pairs, offs)
    with pytest.raises(_capi.SaError, match=re.escape(what)) as e:
        ops.validate_csr(pairs, offs, T, T, BS)
    assert e.value.code == _capi.SA_ERR_CSR


def test_backend_rejects_caller_csr_and_accepts_compiled():
    q, k, v = workloads.seeded_qkv(1, 1, H, H, T, T, D, device=DEV, dtype=torch.bfloat16)
    pairs, offs = _good()
    be = sa.get_backend("cuda_sm100")
    md = PatternMetadata(kind="mask", block_size=BS, block_pairs=pairs, block_pair_offsets=offs)
    be.forward(q, k, v, md)                       # valid caller CSR: validated once, then run
    pairs[0, 1], pairs[0, 2] = 1, 0               # in-place change: validated again, rejected
    with pytest.raises(_capi.SaError) as e:
        be.forward(q, k, v, md)
    assert e.value.code == _capi.SA_ERR_CSR
    out = be.forward(q, k, v, sa.BigBirdKeepRatioPattern(layouts=[(128, 1, 2, 1)], n_heads=H).build(q, k))
    assert bool(torch.isfinite(out).all())
    assert _capi.device_error() == 0
