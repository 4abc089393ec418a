"""Torch-facing wrappers of the C ABI and the ``cuda_sparse_attention`` op namespace.

The reference reserves ``TORCH_LIBRARY(cuda_sparse_attention)`` for its native
ops (kernels/cuda/src/csrc/bind.cu:10-19; wrappers kernels/cuda/src/torch_wrappers/ops.py).
This module adds the B200 ops to that namespace as a FRAGMENT, each a thin
call into ``libsa_b200.so``:

    torch.ops.cuda_sparse_attention.sparse_attn(q, k, v, block_pairs, block_pair_offsets, block_size)
    torch.ops.cuda_sparse_attention.prefill_fwd(...)
    torch.ops.cuda_sparse_attention.decode_fwd(..., n_split)
    torch.ops.cuda_sparse_attention.compile_block_bitmap(bitmap)
    torch.ops.cuda_sparse_attention.compile_token_mask(mask, block_size)
    torch.ops.cuda_sparse_attention.compile_kv_block_list(kv_block_list)
    torch.ops.cuda_sparse_attention.compile_bigbird(layouts, n_heads, T_q, T_k, block_size, variant, like)

The plain functions below are the same entry points without dispatcher
overhead; the backend uses them. Nothing here has a CPU path: non-CUDA
tensors raise.
"""
from __future__ import annotations

import ctypes
import math
from typing import Sequence

import torch

from . import _capi

_NUM_SMS: dict[int, int] = {}


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _num_sms(device: torch.device) -> int:
    idx = device.index if device.index is not None else torch.cuda.current_device()
    if idx not in _NUM_SMS:
        _NUM_SMS[idx] = torch.cuda.get_device_properties(idx).multi_processor_count
    return _NUM_SMS[idx]


def _require_cuda(*ts: torch.Tensor) -> None:
    for t in ts:
        if not t.is_cuda:
            raise RuntimeError("cuda_sparse_attention ops need CUDA tensors (there is no CPU path)")


# ---------------------------------------------------------------------------
# pattern compiler
# ---------------------------------------------------------------------------
def _csr_finish(offsets: torch.Tensor, width: int | None) -> int:
    """Width of block_pairs: the reference's max nnz over heads (one host read),
    or a caller-provided upper bound (no synchronisation)."""
    if width is not None:
        return max(1, int(width))
    return max(1, int(offsets[:, -1].max().item()))


def compile_bigbird(layouts: Sequence[Sequence[int]], n_heads: int, T_q: int, T_k: int, block_size: int,
                    *, variant: int = _capi.SA_BIGBIRD, device: torch.device | str = "cuda",
                    width: int | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """BigBird layouts (one (bs, g, w, r) per KV group) -> (block_pairs [H, W], offsets [H, NQB+1]).

    Bit-exact with BigBird*Pattern._get_block_pairs (bigbird_pattern.py:212-271,
    533-583, 697-753). ``width=None`` reproduces the reference's exact width
    (one device->host read); a given ``width`` must bound every head's nnz.
    """
    device = torch.device(device)
    lib = _capi.load()
    n = len(layouts)
    arr = (_capi.BigBirdLayout * n)(*[_capi.BigBirdLayout(*map(int, l)) for l in layouts])
    nqb = math.ceil(T_q / block_size)
    offsets = torch.empty(n_heads, nqb + 1, dtype=torch.int32, device=device)
    with torch.cuda.device(device):
        s = _stream(device)
        _capi.check(lib.sa_bigbird_offsets(arr, n, n_heads, T_q, T_k, block_size, variant, offsets.data_ptr(), s))
        w = _csr_finish(offsets, width)
        pairs = torch.empty(n_heads, w, dtype=torch.int32, device=device)
        _capi.check(lib.sa_bigbird_pairs(arr, n, n_heads, T_q, T_k, block_size, variant, offsets.data_ptr(),
                                         pairs.data_ptr(), w, s))
    return pairs, offsets


def compile_block_bitmap(bitmap: torch.Tensor, *, width: int | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """Block bitmap [H, NQB, NKB] (nonzero = keep) -> CSR, as build_block_pairs_from_mask's
    CSR loop (patterns/base.py:75-89)."""
    _require_cuda(bitmap)
    bm = bitmap.to(torch.uint8).contiguous()
    H, nqb, nkb = bm.shape
    lib = _capi.load()
    offsets = torch.empty(H, nqb + 1, dtype=torch.int32, device=bm.device)
    with torch.cuda.device(bm.device):
        s = _stream(bm.device)
        _capi.check(lib.sa_bitmap_offsets(bm.data_ptr(), H, nqb, nkb, offsets.data_ptr(), s))
        w = _csr_finish(offsets, width)
        pairs = torch.empty(H, w, dtype=torch.int32, device=bm.device)
        _capi.check(lib.sa_bitmap_pairs(bm.data_ptr(), H, nqb, nkb, offsets.data_ptr(), pairs.data_ptr(), w, s))
    return pairs, offsets


def block_bitmap_from_token_mask(mask: torch.Tensor, block_size: int) -> torch.Tensor:
    """Token mask [H, T_q, T_k] bool -> block bitmap [H, NQB, NKB] uint8 (patterns/base.py:58-73)."""
    _require_cuda(mask)
    m = mask.contiguous()
    if m.dtype != torch.bool and m.dtype != torch.uint8:
        m = m != 0
    H, T_q, T_k = m.shape
    nqb, nkb = math.ceil(T_q / block_size), math.ceil(T_k / block_size)
    bm = torch.empty(H, nqb, nkb, dtype=torch.uint8, device=m.device)
    with torch.cuda.device(m.device):
        _capi.check(_capi.load().sa_block_bitmap_from_token_mask(m.data_ptr(), H, T_q, T_k, block_size,
                                                                 bm.data_ptr(), _stream(m.device)))
    return bm


def compile_token_mask(mask: torch.Tensor, block_size: int) -> tuple[torch.Tensor, torch.Tensor]:
    """build_block_pairs_from_mask (patterns/base.py:36-89) on the device."""
    return compile_block_bitmap(block_bitmap_from_token_mask(mask, block_size))


def compile_kv_block_list(kv_block_list: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """kv_block_list_to_pairs (patterns/base.py:92-133) on the device."""
    _require_cuda(kv_block_list)
    kvl = kv_block_list.to(torch.int32).contiguous()
    H, nqb, mk = kvl.shape
    lib = _capi.load()
    offsets = torch.empty(H, nqb + 1, dtype=torch.int32, device=kvl.device)
    with torch.cuda.device(kvl.device):
        s = _stream(kvl.device)
        _capi.check(lib.sa_kvlist_offsets(kvl.data_ptr(), H, nqb, mk, offsets.data_ptr(), s))
        w = _csr_finish(offsets, None)
        pairs = torch.empty(H, w, dtype=torch.int32, device=kvl.device)
        _capi.check(lib.sa_kvlist_pairs(kvl.data_ptr(), H, nqb, mk, offsets.data_ptr(), pairs.data_ptr(), w, s))
    return pairs, offsets


# ---------------------------------------------------------------------------
# attention
# ---------------------------------------------------------------------------
def _as_bf16(t: torch.Tensor) -> torch.Tensor:
    if t.dtype != torch.bfloat16:
        t = t.to(torch.bfloat16)
    if t.stride(-1) != 1:
        t = t.contiguous()
    return t


def _fill_args(q, k, v, out, pairs, offsets, block_size: int, scale: float | None) -> _capi.AttnArgs:
    B, Hq, T_q, D = q.shape
    Bk, Hkv, T_k, Dk = k.shape
    if v.shape != k.shape or Bk != B or Dk != D:
        raise ValueError(f"shape mismatch q{tuple(q.shape)} k{tuple(k.shape)} v{tuple(v.shape)}")
    if Hq % Hkv:
        raise ValueError(f"Hq={Hq} is not a multiple of Hkv={Hkv}")
    if pairs.dtype != torch.int32 or offsets.dtype != torch.int32:
        raise TypeError("block_pairs / block_pair_offsets must be int32")
    nqb = math.ceil(T_q / block_size)
    if pairs.dim() != 2 or offsets.dim() != 2 or pairs.size(0) != Hq or offsets.size(0) != Hq:
        raise ValueError(f"CSR head dim must be Hq={Hq} (pairs {tuple(pairs.shape)}, offsets {tuple(offsets.shape)})")
    if offsets.size(1) != nqb + 1:
        raise ValueError(f"offsets must be [Hq, {nqb + 1}] for T_q={T_q}, block_size={block_size}; "
                         f"got {tuple(offsets.shape)}")
    if pairs.stride(1) != 1 or offsets.stride(1) != 1 or offsets.stride(0) != nqb + 1:
        raise ValueError("CSR tensors must be row-contiguous")
    a = _capi.AttnArgs()
    a.q, a.k, a.v, a.out = q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr()
    a.pairs, a.offsets = pairs.data_ptr(), offsets.data_ptr()
    for dst, t in ((a.q_strides, q), (a.k_strides, k), (a.v_strides, v), (a.o_strides, out)):
        dst[0], dst[1], dst[2] = t.stride(0), t.stride(1), t.stride(2)
    a.B, a.Hq, a.Hkv, a.T_q, a.T_k, a.D = B, Hq, Hkv, T_q, T_k, D
    a.block_size = block_size
    a.pairs_stride = pairs.stride(0)
    a.scale = float(scale) if scale is not None else 1.0 / math.sqrt(D)
    a.num_sms = _num_sms(q.device)
    return a


def prefill_fwd(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, block_pairs: torch.Tensor,
                block_pair_offsets: torch.Tensor, block_size: int, *, scale: float | None = None,
                out: torch.Tensor | None = None) -> torch.Tensor:
    """Block-sparse attention forward on tcgen05 (replaces universal_sparse_attn,
    kernels/triton/universal_sparse_attn.py:164-238). q [B,Hq,T_q,D]; k/v [B,Hkv,T_k,D]
    (Hkv divides Hq: GQA without repeat_kv). Computes in bf16 with fp32 softmax."""
    _require_cuda(q, k, v, block_pairs, block_pair_offsets)
    in_dtype = q.dtype
    qb, kb, vb = _as_bf16(q), _as_bf16(k), _as_bf16(v)
    o = out if (out is not None and out.dtype == torch.bfloat16) else torch.empty(qb.shape, dtype=torch.bfloat16,
                                                                                 device=q.device)
    a = _fill_args(qb, kb, vb, o, block_pairs, block_pair_offsets, block_size, scale)
    with torch.cuda.device(q.device):
        _capi.check(_capi.load().sa_prefill_fwd(ctypes.byref(a), _stream(q.device)))
    if out is not None and out is not o:
        out.copy_(o)
        return out
    return o if in_dtype == torch.bfloat16 else o.to(in_dtype)


def default_n_split(q: torch.Tensor, k: torch.Tensor) -> int:
    # One CTA per (b, kv head) already fills the GPU once there are ~#SMs of
    # them (measured: more splits only repeat the per-CTA union build).
    B, Hkv = k.shape[0], k.shape[1]
    target = _num_sms(q.device)
    return int(min(64, max(1, math.ceil(target / max(1, B * Hkv)))))


def decode_fwd(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, block_pairs: torch.Tensor,
               block_pair_offsets: torch.Tensor, block_size: int, *, scale: float | None = None,
               n_split: int | None = None, out: torch.Tensor | None = None,
               workspace: tuple[torch.Tensor, torch.Tensor] | None = None) -> torch.Tensor:
    """Split-KV sparse decode (T_q == 1): q [B,Hq,1,D], KV cache [B,Hkv,T_k,D] (any
    T stride, e.g. a view of a larger pre-allocated cache)."""
    _require_cuda(q, k, v, block_pairs, block_pair_offsets)
    in_dtype = q.dtype
    qb, kb, vb = _as_bf16(q), _as_bf16(k), _as_bf16(v)
    B, Hq, _, D = qb.shape
    ns = n_split if n_split is not None else default_n_split(qb, kb)
    o = out if (out is not None and out.dtype == torch.bfloat16) else torch.empty(qb.shape, dtype=torch.bfloat16,
                                                                                 device=q.device)
    if workspace is None:
        po = torch.empty(B * Hq * ns * D, dtype=torch.float32, device=q.device)
        pml = torch.empty(B * Hq * ns * 2, dtype=torch.float32, device=q.device)
    else:
        po, pml = workspace
        if po.numel() < B * Hq * ns * D or pml.numel() < B * Hq * ns * 2:
            raise ValueError("decode workspace too small")
    a = _fill_args(qb, kb, vb, o, block_pairs, block_pair_offsets, block_size, scale)
    with torch.cuda.device(q.device):
        _capi.check(_capi.load().sa_decode_fwd(ctypes.byref(a), ns, po.data_ptr(), pml.data_ptr(),
                                               _stream(q.device)))
    if out is not None and out is not o:
        out.copy_(o)
        return out
    return o if in_dtype == torch.bfloat16 else o.to(in_dtype)


def sparse_attn(q, k, v, block_pairs, block_pair_offsets, block_size: int, *, scale: float | None = None):
    """Decode kernel for T_q == 1, tcgen05 prefill kernel otherwise."""
    if q.size(2) == 1:
        return decode_fwd(q, k, v, block_pairs, block_pair_offsets, block_size, scale=scale)
    return prefill_fwd(q, k, v, block_pairs, block_pair_offsets, block_size, scale=scale)


# ---------------------------------------------------------------------------
# torch.library registration (namespace of kernels/cuda/src/csrc/bind.cu:10)
# ---------------------------------------------------------------------------
_LIB = torch.library.Library("cuda_sparse_attention", "FRAGMENT")
_LIB.define("sparse_attn(Tensor q, Tensor k, Tensor v, Tensor block_pairs, Tensor block_pair_offsets, "
            "int block_size, float? scale=None) -> Tensor")
_LIB.define("prefill_fwd(Tensor q, Tensor k, Tensor v, Tensor block_pairs, Tensor block_pair_offsets, "
            "int block_size, float? scale=None) -> Tensor")
_LIB.define("decode_fwd(Tensor q, Tensor k, Tensor v, Tensor block_pairs, Tensor block_pair_offsets, "
            "int block_size, float? scale=None, int? n_split=None) -> Tensor")
_LIB.define("compile_block_bitmap(Tensor bitmap) -> (Tensor, Tensor)")
_LIB.define("compile_token_mask(Tensor mask, int block_size) -> (Tensor, Tensor)")
_LIB.define("compile_kv_block_list(Tensor kv_block_list) -> (Tensor, Tensor)")
_LIB.define("compile_bigbird(int[] layouts, int n_heads, int T_q, int T_k, int block_size, int variant, "
            "Tensor like) -> (Tensor, Tensor)")


def _op_sparse_attn(q, k, v, p, o, bs, scale=None):
    return sparse_attn(q, k, v, p, o, bs, scale=scale)


def _op_prefill(q, k, v, p, o, bs, scale=None):
    return prefill_fwd(q, k, v, p, o, bs, scale=scale)


def _op_decode(q, k, v, p, o, bs, scale=None, n_split=None):
    return decode_fwd(q, k, v, p, o, bs, scale=scale, n_split=n_split)


def _op_bigbird(layouts, n_heads, T_q, T_k, bs, variant, like):
    lay = [tuple(layouts[i:i + 4]) for i in range(0, len(layouts), 4)]
    return compile_bigbird(lay, n_heads, T_q, T_k, bs, variant=variant, device=like.device)


_LIB.impl("sparse_attn", _op_sparse_attn, "CUDA")
_LIB.impl("prefill_fwd", _op_prefill, "CUDA")
_LIB.impl("decode_fwd", _op_decode, "CUDA")
_LIB.impl("compile_block_bitmap", compile_block_bitmap, "CUDA")
_LIB.impl("compile_token_mask", compile_token_mask, "CUDA")
_LIB.impl("compile_kv_block_list", compile_kv_block_list, "CUDA")
_LIB.impl("compile_bigbird", _op_bigbird, "CUDA")

for _name in ("sparse_attn", "prefill_fwd", "decode_fwd"):
    def _fake(q, k, v, p, o, bs, scale=None, n_split=None):  # noqa: ARG001
        return torch.empty_like(q)
    torch.library.register_fake(f"cuda_sparse_attention::{_name}", _fake, lib=_LIB)
