"""The allocation-free decode entry point (sa_decode_fwd_noalloc).

Some callers cannot allocate device memory when they call the decode kernel
(a plugin that lives inside another framework's memory pool, or a serving loop
that must not allocate once it runs). For them the library keeps the split
partials in its own fixed device array. These tests call that entry point
through the C ABI and check it against sa_decode_fwd with caller-provided
scratch, on two calls in a row (the array keeps the previous call's contents).

The file name makes pytest collect it last.
"""
from __future__ import annotations

import ctypes
import math

import pytest
import torch

from sparseattentioninfer_b200 import _capi, ops, workloads

DEV = "cuda:0"
MAX_ABS = 2e-2
MEAN_ABS = 2e-3


def _decode_case(seed: int, B: int, Hq: int, Hkv: int, T_k: int, D: int, layouts):
    q, k, v = workloads.seeded_qkv(seed, B, Hq, Hkv, 1, T_k, D, device=DEV, dtype=torch.bfloat16)
    pairs, offs = ops.compile_bigbird(layouts, Hq, 1, T_k, layouts[0][0], device=DEV)
    return q, k, v, pairs, offs


def _call_noalloc(q, k, v, pairs, offs, bs, n_split):
    out = torch.empty_like(q)
    args = ops._fill_args(q, k, v, out, pairs, offs, bs, None)
    lib = _capi.load()
    stream = torch.cuda.current_stream().cuda_stream
    _capi.check(lib.sa_decode_fwd_noalloc(ctypes.byref(args), n_split, stream))
    return out


@pytest.mark.gpu
def test_noalloc_matches_caller_scratch_twice():
    cases = [
        # seed, B, Hq, Hkv, T_k, D, layouts, n_split
        (1, 4, 32, 8, 3000, 128, [(64, 2, 4, 2)], 3),
        (2, 2, 8, 8, 777, 64, [(64, 1, 3, 1)], 5),
        (4, 3, 16, 4, 1500, 128, [(64, 2, 4, 2)], 1),   # one split: output written directly
    ]
    for seed, B, Hq, Hkv, T_k, D, layouts, ns in cases:
        q, k, v, pairs, offs = _decode_case(seed, B, Hq, Hkv, T_k, D, layouts)
        bs = layouts[0][0]
        ref = ops.decode_fwd(q, k, v, pairs, offs, bs, n_split=ns)
        for _ in range(2):  # second call sees the first call's leftovers in the shared array
            got = _call_noalloc(q, k, v, pairs, offs, bs, ns)
            torch.cuda.synchronize()
            err = (got.float() - ref.float()).abs()
            assert torch.isfinite(got.float()).all()
            assert err.max().item() <= MAX_ABS and err.mean().item() <= MEAN_ABS, err.max().item()
    assert _capi.device_error() == 0


@pytest.mark.gpu
def test_noalloc_rejects_requests_beyond_the_array():
    B, Hq, Hkv, T_k, D = 64, 64, 8, 1024, 128
    q, k, v, pairs, offs = _decode_case(3, 1, Hq, Hkv, T_k, D, [(64, 2, 4, 2)])
    q = q.expand(B, -1, -1, -1).contiguous()
    k = k.expand(B, -1, -1, -1).contiguous()
    v = v.expand(B, -1, -1, -1).contiguous()
    n_split = 64  # B*Hq*n_split*(D+2) = 34 M floats > 4 M
    assert B * Hq * n_split * (D + 2) > 4 * 1024 * 1024
    with pytest.raises(_capi.SaError, match="decode scratch needs"):
        _call_noalloc(q, k, v, pairs, offs, 64, n_split)
    assert math.isfinite(float(q.float().sum()))


@pytest.mark.gpu
def test_noalloc_one_split_has_no_size_limit():
    """With n_split == 1 the array is not used, so shapes beyond it still run."""
    B, Hq, Hkv, T_k, D = 256, 64, 8, 1024, 128
    q, k, v, pairs, offs = _decode_case(5, 1, Hq, Hkv, T_k, D, [(64, 2, 4, 2)])
    q = q.expand(B, -1, -1, -1).contiguous()
    k = k.expand(B, -1, -1, -1).contiguous()
    v = v.expand(B, -1, -1, -1).contiguous()
    assert B * Hq * 2 * (D + 2) > 4 * 1024 * 1024  # n_split = 2 would not fit
    ref = ops.decode_fwd(q, k, v, pairs, offs, 64, n_split=1)
    got = _call_noalloc(q, k, v, pairs, offs, 64, 1)
    torch.cuda.synchronize()
    assert torch.equal(got, ref)
    assert _capi.device_error() == 0
