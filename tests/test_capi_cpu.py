"""C-ABI library: loads without a GPU, exports every symbol the header declares,
and rejects bad arguments on the host before touching the device."""
from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

from sparseattentioninfer_b200 import _capi

HEADER = Path(__file__).resolve().parents[1] / "include" / "sparse_attn_b200.h"


def header_symbols() -> set[str]:
    text = HEADER.read_text()
    return set(re.findall(r"^\s*(?:SA_API\s+)?(?:int|const char\*)\s+(sa_\w+)\s*\(", text, flags=re.M))


def test_exports_match_header():
    lib = _capi.load()
    syms = header_symbols()
    assert syms == set(_capi.EXPORTED), syms ^ set(_capi.EXPORTED)
    for s in syms:
        assert hasattr(lib, s), s


def test_version_and_empty_error():
    assert "sm_100a" in _capi.version()


def test_prefill_rejects_null_args():
    lib = _capi.load()
    assert lib.sa_prefill_fwd(None, None) == _capi.SA_ERR_INVALID
    assert b"NULL" in lib.sa_last_error()


def _args(**over):
    a = _capi.AttnArgs()
    fake = 1 << 20  # never dereferenced: validation fails before any launch
    a.q = a.k = a.v = a.out = a.pairs = a.offsets = fake
    for arr in (a.q_strides, a.k_strides, a.v_strides, a.o_strides):
        arr[0], arr[1], arr[2] = 32 * 128 * 128, 128 * 128, 128
    a.B, a.Hq, a.Hkv, a.T_q, a.T_k, a.D, a.block_size, a.pairs_stride, a.scale = 1, 32, 8, 128, 128, 128, 64, 4, 0.1
    for k, v in over.items():
        setattr(a, k, v)
    return a


@pytest.mark.parametrize("field,value,code", [
    ("D", 96, _capi.SA_ERR_UNSUPPORTED),
    ("block_size", 48, _capi.SA_ERR_INVALID),
    ("block_size", 8, _capi.SA_ERR_INVALID),
    ("Hkv", 5, _capi.SA_ERR_INVALID),
    ("T_q", 256, _capi.SA_ERR_INVALID),
    ("B", 0, _capi.SA_ERR_INVALID),
    ("q", (1 << 20) + 8, _capi.SA_ERR_INVALID),
])
def test_prefill_host_validation(field, value, code):
    lib = _capi.load()
    a = _args(**{field: value})
    assert lib.sa_prefill_fwd(ctypes.byref(a), None) == code
    assert lib.sa_last_error()


def test_decode_host_validation():
    lib = _capi.load()
    a = _args(T_q=1)
    assert lib.sa_decode_fwd(ctypes.byref(a), 0, 1, 1, None) == _capi.SA_ERR_INVALID  # n_split 0
    a = _args(T_q=2)
    assert lib.sa_decode_fwd(ctypes.byref(a), 2, 1, 1, None) == _capi.SA_ERR_INVALID  # T_q != 1
    a = _args(T_q=1, Hq=48, Hkv=4)
    assert lib.sa_decode_fwd(ctypes.byref(a), 2, 1, 1, None) == _capi.SA_ERR_UNSUPPORTED  # group 12
    a = _args(T_q=1, T_k=64 * 8193, block_size=64)
    assert lib.sa_decode_fwd(ctypes.byref(a), 1, 1, 1, None) == _capi.SA_ERR_UNSUPPORTED  # NKB > 8192
    assert b"8192" in lib.sa_last_error()
    a = _args(T_q=1, T_k=64 * 4096, block_size=64, pairs_stride=4096)
    assert lib.sa_decode_fwd(ctypes.byref(a), 1, 1, 1, None) == _capi.SA_ERR_UNSUPPORTED  # union > 2048
    assert b"2048" in lib.sa_last_error()


def test_noalloc_host_validation_matches_decode():
    """The allocation-free entry point returns the same error codes as sa_decode_fwd."""
    lib = _capi.load()
    for kw in ({"D": 96}, {"T_q": 2}, {"B": 0}):
        a = _args(**{"T_q": 1, **kw})
        assert lib.sa_decode_fwd_noalloc(ctypes.byref(a), 1, None) == lib.sa_decode_fwd(ctypes.byref(a), 1, 1, 1,
                                                                                         None)


def test_pattern_host_validation():
    lib = _capi.load()
    lay = (_capi.BigBirdLayout * 3)(*[_capi.BigBirdLayout(64, 1, 2, 0)] * 3)
    assert lib.sa_bigbird_offsets(lay, 3, 8, 128, 128, 64, 0, 1 << 20, None) == _capi.SA_ERR_INVALID
    assert lib.sa_bigbird_offsets(lay, 1, 8, 256, 128, 64, 0, 1 << 20, None) == _capi.SA_ERR_INVALID
    assert lib.sa_bigbird_offsets(lay, 1, 8, 128, 128, 64, 7, 1 << 20, None) == _capi.SA_ERR_INVALID
    assert lib.sa_block_bitmap_from_token_mask(1 << 20, 1, 16, 16, 24, 1 << 20, None) == _capi.SA_ERR_INVALID


def test_package_import_exposes_reference_api():
    import sparseattentioninfer_b200 as sa
    b = sa.get_backend("cuda_sm100")
    assert b.actual_backend == "cuda_sm100"
    with pytest.raises(ValueError):
        sa.get_backend("triton_universal")
    reg = sa.register_with_reference({})
    assert reg["cuda_sm100"] is sa.CudaSm100Backend


def test_validate_csr_host_arguments():
    lib = _capi.load()
    assert lib.sa_validate_csr(None, None, 1, 1, 1, 1, None, None) == _capi.SA_ERR_INVALID
    assert lib.sa_validate_csr(1 << 20, 1 << 20, 0, 1, 1, 1, 1 << 20, None) == _capi.SA_ERR_INVALID


def test_attention_backend_is_abstract():
    import sparseattentioninfer_b200 as sa
    with pytest.raises(TypeError):
        sa.AttentionBackend()
    assert "forward" in sa.AttentionBackend.__abstractmethods__


def test_linear_m8_host_validation():
    """sa_linear_m8 rejects unsupported shapes and layouts before any CUDA call."""
    lib = _capi.load()
    P = 1 << 20  # a 16-byte aligned dummy address (never dereferenced: the checks fail first)
    ok = dict(x=P, M=8, K=4096, xs=4096, w=P, N=768, ws=4096, o=P, os=768, glu=0)

    def call(**kw):
        a = {**ok, **kw}
        return lib.sa_linear_m8(a["x"], a["M"], a["K"], a["xs"], a["w"], a["N"], a["ws"], a["o"], a["os"],
                                a["glu"], None)

    assert call(x=None) == _capi.SA_ERR_INVALID
    assert call(M=9) == _capi.SA_ERR_UNSUPPORTED and b"tokens" in lib.sa_last_error()
    assert call(M=0) == _capi.SA_ERR_UNSUPPORTED
    assert call(K=4000) == _capi.SA_ERR_UNSUPPORTED
    assert call(N=770) == _capi.SA_ERR_UNSUPPORTED
    assert call(x=P + 8) == _capi.SA_ERR_INVALID  # rows not on 16-byte boundaries
    assert call(xs=4100) == _capi.SA_ERR_INVALID
    assert call(ws=2048) == _capi.SA_ERR_INVALID  # stride shorter than K
