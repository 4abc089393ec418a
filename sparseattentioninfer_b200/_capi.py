"""ctypes binding of the C ABI declared in ``include/sparse_attn_b200.h``.

The shared library is built in-tree (``_lib/libsa_b200.so``). There is no
fallback: if the library is missing or fails to load, every entry point raises.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

_PKG = Path(__file__).resolve().parent
LIB_PATH = _PKG / "_lib" / "libsa_b200.so"

# Every symbol include/sparse_attn_b200.h declares (checked by the CPU tests).
EXPORTED = (
    "sa_version",
    "sa_last_error",
    "sa_device_error",
    "sa_bigbird_offsets",
    "sa_bigbird_pairs",
    "sa_bigbird_decode_row",
    "sa_block_bitmap_from_token_mask",
    "sa_bitmap_offsets",
    "sa_bitmap_pairs",
    "sa_validate_csr",
    "sa_kvlist_offsets",
    "sa_kvlist_pairs",
    "sa_prefill_fwd",
    "sa_decode_fwd",
    "sa_decode_fwd_seqlen",
    "sa_decode_fwd_noalloc",
    "sa_qk_norm_rope_append",
    "sa_add_rms_norm",
    "sa_silu_mul",
    "sa_linear_m8",
    "sa_topk_softmax_pv",
    "sa_ar_alloc",
    "sa_ar_free",
    "sa_ar_ipc_handle",
    "sa_ar_ipc_open",
    "sa_ar_ipc_close",
    "sa_allreduce_add_rms_norm",
)

SA_OK = 0
SA_ERR_INVALID = -1
SA_ERR_UNSUPPORTED = -2
SA_ERR_CUDA = -3
SA_ERR_TIMEOUT = -4
SA_ERR_CSR = -5
SA_BIGBIRD = 0
SA_BIGBIRD2 = 1

_c_i32 = ctypes.c_int32
_c_i64 = ctypes.c_int64
_c_p = ctypes.c_void_p


class SaError(RuntimeError):
    """Raised when a C ABI call returns a non-zero status."""

    def __init__(self, code: int, msg: str):
        super().__init__(f"[sa error {code}] {msg}")
        self.code = code


class BigBirdLayout(ctypes.Structure):
    _fields_ = [("block_size", _c_i32), ("global_blocks", _c_i32), ("sliding_blocks", _c_i32),
                ("random_blocks", _c_i32)]


class AttnArgs(ctypes.Structure):
    _fields_ = [
        ("q", _c_p), ("k", _c_p), ("v", _c_p), ("out", _c_p), ("pairs", _c_p), ("offsets", _c_p),
        ("q_strides", _c_i64 * 3), ("k_strides", _c_i64 * 3), ("v_strides", _c_i64 * 3),
        ("o_strides", _c_i64 * 3),
        ("B", _c_i32), ("Hq", _c_i32), ("Hkv", _c_i32), ("T_q", _c_i32), ("T_k", _c_i32), ("D", _c_i32),
        ("block_size", _c_i32), ("pairs_stride", _c_i32), ("scale", ctypes.c_float), ("num_sms", _c_i32),
    ]


class QkvPrologueArgs(ctypes.Structure):
    _fields_ = [
        ("qkv", _c_p), ("qkv_sb", _c_i64), ("qkv_st", _c_i64), ("q_weight", _c_p), ("k_weight", _c_p),
        ("cos", _c_p), ("sin", _c_p), ("q_out", _c_p), ("q_strides", _c_i64 * 3), ("k_cache", _c_p),
        ("k_strides", _c_i64 * 3), ("v_cache", _c_p), ("v_strides", _c_i64 * 3),
        ("B", _c_i32), ("T", _c_i32), ("Hq", _c_i32), ("Hkv", _c_i32), ("D", _c_i32), ("capacity", _c_i32),
        ("pos", _c_i32), ("pos_dev", _c_p), ("eps", ctypes.c_float),
    ]


class TopkArgs(ctypes.Structure):
    _fields_ = [("scores", _c_p), ("s_row", _c_i64), ("v", _c_p), ("v_strides", _c_i64 * 3), ("out", _c_p),
                ("o_strides", _c_i64 * 3), ("out_f32", _c_i32), ("B", _c_i32), ("Hkv", _c_i32), ("G", _c_i32),
                ("rows_per_head", _c_i32), ("t0", _c_i32), ("T_q", _c_i32), ("T_k", _c_i32), ("D", _c_i32),
                ("top_k", _c_i32)]


class ArPeers(ctypes.Structure):
    _fields_ = [("rank", _c_i32), ("world", _c_i32), ("data", _c_p * 8), ("flags", _c_p * 8), ("epoch", _c_p),
                ("max_ctas", _c_i32)]


_lib = None


def load(path: str | os.PathLike | None = None) -> ctypes.CDLL:
    """Load (once) and return the C-ABI library; raises if it is absent.
    ``SA_LIBRARY`` overrides the path (e.g. an instrumented debug build)."""
    global _lib
    if _lib is not None:
        return _lib
    p = Path(path) if path is not None else Path(os.environ.get("SA_LIBRARY", LIB_PATH))
    if not p.exists():
        raise ImportError(
            f"sparseattentioninfer_b200 C library not found at {p}; build it with "
            "`python sparseattentioninfer_b200/_build.py` (no CPU fallback exists)")
    lib = ctypes.CDLL(str(p))
    lib.sa_version.restype = ctypes.c_char_p
    lib.sa_last_error.restype = ctypes.c_char_p
    lib.sa_device_error.argtypes = [ctypes.POINTER(_c_i32)]
    lay = ctypes.POINTER(BigBirdLayout)
    lib.sa_bigbird_offsets.argtypes = [lay, _c_i32, _c_i32, _c_i32, _c_i32, _c_i32, _c_i32, _c_p, _c_p]
    lib.sa_bigbird_pairs.argtypes = [lay, _c_i32, _c_i32, _c_i32, _c_i32, _c_i32, _c_i32, _c_p, _c_p, _c_i32, _c_p]
    lib.sa_bigbird_decode_row.argtypes = [lay, _c_i32, _c_i32, _c_i32, _c_i32, _c_p, _c_i32, _c_i32, _c_p, _c_p,
                                          _c_i32, _c_p]
    lib.sa_block_bitmap_from_token_mask.argtypes = [_c_p, _c_i32, _c_i32, _c_i32, _c_i32, _c_p, _c_p]
    lib.sa_bitmap_offsets.argtypes = [_c_p, _c_i32, _c_i32, _c_i32, _c_p, _c_p]
    lib.sa_bitmap_pairs.argtypes = [_c_p, _c_i32, _c_i32, _c_i32, _c_p, _c_p, _c_i32, _c_p]
    lib.sa_validate_csr.argtypes = [_c_p, _c_p, _c_i32, _c_i32, _c_i32, _c_i32, _c_p, _c_p]
    lib.sa_kvlist_offsets.argtypes = [_c_p, _c_i32, _c_i32, _c_i32, _c_p, _c_p]
    lib.sa_kvlist_pairs.argtypes = [_c_p, _c_i32, _c_i32, _c_i32, _c_p, _c_p, _c_i32, _c_p]
    lib.sa_prefill_fwd.argtypes = [ctypes.POINTER(AttnArgs), _c_p]
    lib.sa_decode_fwd.argtypes = [ctypes.POINTER(AttnArgs), _c_i32, _c_p, _c_p, _c_p]
    lib.sa_decode_fwd_seqlen.argtypes = [ctypes.POINTER(AttnArgs), _c_p, _c_i32, _c_p, _c_p, _c_p]
    lib.sa_qk_norm_rope_append.argtypes = [ctypes.POINTER(QkvPrologueArgs), _c_p]
    lib.sa_add_rms_norm.argtypes = [_c_p, _c_p, _c_p, _c_p, _c_i64, _c_i32, _c_i64, _c_i64, _c_i64, ctypes.c_float,
                                    _c_p]
    lib.sa_silu_mul.argtypes = [_c_p, _c_p, _c_i64, _c_i32, _c_i64, _c_i64, _c_p]
    lib.sa_linear_m8.argtypes = [_c_p, _c_i32, _c_i32, _c_i64, _c_p, _c_i32, _c_i64, _c_p, _c_i64, _c_i32, _c_p]
    lib.sa_topk_softmax_pv.argtypes = [ctypes.POINTER(TopkArgs), _c_p]
    lib.sa_ar_alloc.argtypes = [ctypes.c_size_t, ctypes.POINTER(_c_p)]
    lib.sa_ar_free.argtypes = [_c_p]
    lib.sa_ar_ipc_handle.argtypes = [_c_p, _c_p]
    lib.sa_ar_ipc_open.argtypes = [_c_p, ctypes.POINTER(_c_p)]
    lib.sa_ar_ipc_close.argtypes = [_c_p]
    lib.sa_allreduce_add_rms_norm.argtypes = [ctypes.POINTER(ArPeers), _c_i64, _c_p, _c_p, _c_p, _c_i64, _c_i32,
                                              _c_i64, _c_i64, ctypes.c_float, _c_p]
    lib.sa_decode_fwd_noalloc.argtypes = [ctypes.POINTER(AttnArgs), _c_i32, _c_p]
    for name in EXPORTED:
        if name not in ("sa_version", "sa_last_error"):
            getattr(lib, name).restype = ctypes.c_int
    _lib = lib
    return lib


def check(rc: int) -> None:
    if rc != SA_OK:
        msg = load().sa_last_error().decode(errors="replace")
        raise SaError(rc, msg)


def version() -> str:
    return load().sa_version().decode()


def device_error() -> int:
    """Read and clear the device error word (synchronises the device)."""
    code = _c_i32(0)
    check(load().sa_device_error(ctypes.byref(code)))
    return int(code.value)
