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
    torch.ops.cuda_sparse_attention.cuda_bigbird_sparse_attention(q, k, v, block_size=64, global_blocks=2,
                                                                  sliding_blocks=3, random_blocks=2)

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



def bigbird_decode_row(layouts, n_heads: int, seq_len: torch.Tensor, block_size: int, pairs: torch.Tensor,
                       offsets: torch.Tensor, *, head_lo: int = 0, variant: int = _capi.SA_BIGBIRD) -> None:
    """Decode rows (T_q = 1) of query heads [head_lo, head_lo + pairs.shape[0]) for the
    key count in ``seq_len`` (int32 device scalar), written into ``pairs``
    [rows, W] and ``offsets`` [rows, 2] on the device (sa_bigbird_decode_row):
    the rows compile_bigbird(layouts, n_heads, 1, T_k, ...) gives, without the
    host knowing T_k (graph-replayed decode)."""
    _require_cuda(seq_len, pairs, offsets)
    if seq_len.dtype != torch.int32 or pairs.dtype != torch.int32 or offsets.dtype != torch.int32:
        raise TypeError("int32 tensors expected")
    rows = pairs.shape[0]
    if offsets.shape != (rows, 2) or not pairs.is_contiguous() or not offsets.is_contiguous():
        raise ValueError("pairs [rows, W] and offsets [rows, 2], contiguous")
    lib = _capi.load()
    n = len(layouts)
    arr = (_capi.BigBirdLayout * n)(*[_capi.BigBirdLayout(*map(int, l)) for l in layouts])
    with torch.cuda.device(pairs.device):
        _capi.check(lib.sa_bigbird_decode_row(arr, n, n_heads, head_lo, rows, seq_len.data_ptr(), block_size, variant,
                                              offsets.data_ptr(), pairs.data_ptr(), pairs.shape[1],
                                              _stream(pairs.device)))


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


def validate_csr(block_pairs: torch.Tensor, block_pair_offsets: torch.Tensor, T_q: int, T_k: int,
                 block_size: int) -> None:
    """Checks a caller-supplied CSR the way the kernels need it (sa_validate_csr):
    offsets start at 0, never decrease and stay within the pairs width; block
    indices lie in [0, ceil(T_k / block_size)) and strictly increase along each
    row. Raises SaError (SA_ERR_CSR) naming the first violation. One device->host
    read."""
    _require_cuda(block_pairs, block_pair_offsets)
    if block_pairs.dtype != torch.int32 or block_pair_offsets.dtype != torch.int32:
        raise TypeError("block_pairs / block_pair_offsets must be int32")
    H = block_pairs.size(0)
    nqb, nkb = math.ceil(T_q / block_size), math.ceil(T_k / block_size)
    if block_pair_offsets.shape != (H, nqb + 1) or block_pairs.stride(1) != 1 or \
            not block_pair_offsets.is_contiguous():
        raise ValueError(f"offsets must be contiguous [H, {nqb + 1}] and pairs row-contiguous")
    res = torch.empty(4, dtype=torch.int32, device=block_pairs.device)
    with torch.cuda.device(block_pairs.device):
        _capi.check(_capi.load().sa_validate_csr(block_pairs.data_ptr(), block_pair_offsets.data_ptr(), H, nqb, nkb,
                                                 block_pairs.stride(0), res.data_ptr(),
                                                 _stream(block_pairs.device)))


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
               workspace: tuple[torch.Tensor, torch.Tensor] | None = None,
               seq_len: torch.Tensor | None = None) -> torch.Tensor:
    """Split-KV sparse decode (T_q == 1): q [B,Hq,1,D], KV cache [B,Hkv,T_k,D] (any
    T stride, e.g. a view of a larger pre-allocated cache).

    ``seq_len`` (int32 device tensor, one element): the live key count is read
    from it on the device and k/v span the capacity, so the call can be captured
    in a CUDA graph and replayed as the cache grows (sa_decode_fwd_seqlen)."""
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
        if seq_len is None:
            _capi.check(_capi.load().sa_decode_fwd(ctypes.byref(a), ns, po.data_ptr(), pml.data_ptr(),
                                                   _stream(q.device)))
        else:
            _require_cuda(seq_len)
            if seq_len.dtype != torch.int32 or seq_len.numel() < 1:
                raise TypeError("seq_len must be an int32 device tensor")
            _capi.check(_capi.load().sa_decode_fwd_seqlen(ctypes.byref(a), seq_len.data_ptr(), ns, po.data_ptr(),
                                                          pml.data_ptr(), _stream(q.device)))
    if out is not None and out is not o:
        out.copy_(o)
        return out
    return o if in_dtype == torch.bfloat16 else o.to(in_dtype)



# ---------------------------------------------------------------------------
# Decoder-layer steps around attention (sa_layer_ops.cu)
# ---------------------------------------------------------------------------
def qk_norm_rope_append(qkv: torch.Tensor, q_weight: torch.Tensor, k_weight: torch.Tensor, cos: torch.Tensor,
                        sin: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, *, Hq: int, Hkv: int,
                        pos: int = 0, pos_dev: torch.Tensor | None = None, eps: float = 1e-6,
                        q_out: torch.Tensor | None = None) -> torch.Tensor:
    """From qkv [B, T, Hq+2*Hkv, D] (the fused projection output): returns
    q = RoPE(RMSNorm(q)) [B, Hq, T, D] (a strided view when ``q_out`` is None) and
    appends RoPE(RMSNorm(k)) and v to the caches [B, Hkv, capacity, D] at
    positions pos.. (``pos_dev``: int32 device scalar read on the device).
    The hook's q_norm/k_norm/apply_rotary_pos_emb/cache update
    (modeling_sparse_qwen3.py:211-231) in one launch."""
    _require_cuda(qkv, q_weight, k_weight, cos, sin, k_cache, v_cache)
    B, T, NH, D = qkv.shape
    if NH != Hq + 2 * Hkv:
        raise ValueError(f"qkv has {NH} heads, expected {Hq}+2*{Hkv}")
    if qkv.stride(3) != 1 or qkv.stride(2) != D:
        raise ValueError("qkv heads must be contiguous [.., heads, D]")
    for t in (qkv, q_weight, k_weight, cos, sin, k_cache, v_cache):
        if t.dtype != torch.bfloat16:
            raise TypeError("bf16 tensors expected")
    if q_out is None:
        q_out = torch.empty(B, T, Hq, D, dtype=torch.bfloat16, device=qkv.device).transpose(1, 2)
    a = _capi.QkvPrologueArgs()
    a.qkv, a.qkv_sb, a.qkv_st = qkv.data_ptr(), qkv.stride(0), qkv.stride(1)
    a.q_weight, a.k_weight = q_weight.data_ptr(), k_weight.data_ptr()
    a.cos, a.sin = cos.data_ptr(), sin.data_ptr()
    a.q_out, a.k_cache, a.v_cache = q_out.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr()
    for dst, t in ((a.q_strides, q_out), (a.k_strides, k_cache), (a.v_strides, v_cache)):
        if t.stride(3) != 1:
            raise ValueError("last dimension must be contiguous")
        dst[0], dst[1], dst[2] = t.stride(0), t.stride(1), t.stride(2)
    a.B, a.T, a.Hq, a.Hkv, a.D, a.capacity = B, T, Hq, Hkv, D, min(k_cache.shape[2], cos.shape[0])
    a.pos = int(pos)
    if pos_dev is not None:
        if pos_dev.dtype != torch.int32:
            raise TypeError("pos_dev must be int32")
        a.pos_dev = pos_dev.data_ptr()
    a.eps = float(eps)
    with torch.cuda.device(qkv.device):
        _capi.check(_capi.load().sa_qk_norm_rope_append(ctypes.byref(a), _stream(qkv.device)))
    return q_out


def add_rms_norm(x: torch.Tensor, y: torch.Tensor | None, weight: torch.Tensor, eps: float = 1e-6,
                 out: torch.Tensor | None = None) -> torch.Tensor:
    """x += y in place (bf16, y may be None), then returns RMSNorm(x) * weight over
    the last dimension (Qwen3RMSNorm after a residual add), rows of x [.., n]."""
    tensors = [x, weight] + ([y] if y is not None else [])
    _require_cuda(*tensors)
    n = x.shape[-1]
    x2 = x.view(-1, n)
    y2 = y.reshape(-1, n) if y is not None else None
    if out is None:
        out = torch.empty_like(x)
    o2 = out.view(-1, n)
    for t in tensors + [out]:
        if t.dtype != torch.bfloat16 or t.stride(-1) != 1:
            raise TypeError("bf16 tensors with a contiguous last dimension expected")
    with torch.cuda.device(x.device):
        _capi.check(_capi.load().sa_add_rms_norm(
            x2.data_ptr(), y2.data_ptr() if y2 is not None else None, weight.data_ptr(), o2.data_ptr(), x2.shape[0],
            n, x2.stride(0), y2.stride(0) if y2 is not None else 0, o2.stride(0), float(eps), _stream(x.device)))
    return out


def silu_mul(gate_up: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """silu(gate_up[..., :I]) * gate_up[..., I:] (Qwen3MLP act_fn(gate) * up)."""
    _require_cuda(gate_up)
    n = gate_up.shape[-1]
    inter = n // 2
    g2 = gate_up.view(-1, n)
    if out is None:
        out = torch.empty(*gate_up.shape[:-1], inter, dtype=gate_up.dtype, device=gate_up.device)
    o2 = out.view(-1, inter)
    if gate_up.dtype != torch.bfloat16 or out.dtype != torch.bfloat16:
        raise TypeError("bf16 tensors expected")
    with torch.cuda.device(gate_up.device):
        _capi.check(_capi.load().sa_silu_mul(g2.data_ptr(), o2.data_ptr(), g2.shape[0], inter, g2.stride(0),
                                             o2.stride(0), _stream(gate_up.device)))
    return out


def linear_m8(x: torch.Tensor, weight: torch.Tensor, out: torch.Tensor | None = None, *,
              glu: bool = False) -> torch.Tensor:
    """x [..., K] (at most 8 rows) times weight [N, K]^T -> [..., N] (nn.Linear
    without bias), one weight-streaming launch (sa_linear_m8). With ``glu`` the
    weight is the fused [gate; up] matrix [2N, K] and the result is
    silu(x W_gate^T) * (x W_up^T) [..., N] (Qwen3MLP's activation fused)."""
    _require_cuda(x, weight)
    if x.dtype != torch.bfloat16 or weight.dtype != torch.bfloat16:
        raise TypeError("bf16 tensors expected")
    K = x.shape[-1]
    x2 = x.reshape(-1, K)
    if x2.stride(-1) != 1 or weight.stride(-1) != 1:
        raise ValueError("x and weight need unit stride in K")
    N = weight.shape[0] // 2 if glu else weight.shape[0]
    if out is None:
        out = torch.empty(*x.shape[:-1], N, dtype=x.dtype, device=x.device)
    o2 = out.view(-1, N)
    if out.dtype != torch.bfloat16 or o2.stride(-1) != 1:
        raise TypeError("out: bf16 with unit stride")
    with torch.cuda.device(x.device):
        _capi.check(_capi.load().sa_linear_m8(x2.data_ptr(), x2.shape[0], K, x2.stride(0), weight.data_ptr(), N,
                                              weight.stride(0), o2.data_ptr(), o2.stride(0), int(bool(glu)),
                                              _stream(x.device)))
    return out



def topk_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, top_k: int, *, scale: float | None = None,
                   max_score_bytes: int = 1 << 29) -> torch.Tensor:
    """Data-dependent top-k attention (the reference's TopKPattern through
    MaskedSdpaBackend, masked_sdpa.py:51-63): per query row, the causal scores'
    top_k entries go through softmax and weight V. Scores are an fp32 GEMM of
    the (bf16-valued) inputs, query rows in chunks of at most
    ``max_score_bytes`` of scores; masking, selection, softmax and the gathered
    PV product are sa_topk_softmax_pv. GQA reads K/V head h // (Hq/Hkv)."""
    _require_cuda(q, k, v)
    B, Hq, T_q, D = q.shape
    Hkv, T_k = k.shape[1], k.shape[2]
    if Hq % Hkv:
        raise ValueError(f"Hq={Hq} is not a multiple of Hkv={Hkv}")
    if T_q > T_k:
        raise ValueError("T_q must not exceed T_k")
    G = Hq // Hkv
    sc = float(scale) if scale is not None else 1.0 / math.sqrt(D)
    qf, kf = q.float(), k.float()
    vb = _as_bf16(v)
    out_f32 = q.dtype == torch.float32
    out = torch.empty(B, Hq, T_q, D, dtype=torch.float32 if out_f32 else torch.bfloat16, device=q.device)
    rows = max(1, min(T_q, max_score_bytes // max(1, B * Hq * T_k * 4)))
    lib = _capi.load()
    for t0 in range(0, T_q, rows):
        rc = min(rows, T_q - t0)
        qc = qf[:, :, t0:t0 + rc].reshape(B, Hkv, G * rc, D)
        scores = torch.matmul(qc, kf.transpose(-1, -2)).mul_(sc).contiguous()
        a = _capi.TopkArgs()
        a.scores, a.s_row = scores.data_ptr(), T_k
        a.v = vb.data_ptr()
        a.v_strides[0], a.v_strides[1], a.v_strides[2] = vb.stride(0), vb.stride(1), vb.stride(2)
        a.out = out.data_ptr()
        a.o_strides[0], a.o_strides[1], a.o_strides[2] = out.stride(0), out.stride(1), out.stride(2)
        a.out_f32 = int(out_f32)
        a.B, a.Hkv, a.G, a.rows_per_head, a.t0, a.T_q, a.T_k, a.D, a.top_k = B, Hkv, G, rc, t0, T_q, T_k, D, top_k
        with torch.cuda.device(q.device):
            _capi.check(lib.sa_topk_softmax_pv(ctypes.byref(a), _stream(q.device)))
    return out if q.dtype in (torch.float32, torch.bfloat16) else out.to(q.dtype)


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
_LIB.define("cuda_bigbird_sparse_attention(Tensor q, Tensor k, Tensor v, int block_size=64, int global_blocks=2, "
            "int sliding_blocks=3, int random_blocks=2) -> Tensor")
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


def cuda_bigbird_sparse_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, block_size: int = 64,
                                  global_blocks: int = 2, sliding_blocks: int = 3,
                                  random_blocks: int = 2) -> torch.Tensor:
    """The op the reference reserves for a native BigBird kernel
    (``cuda_bigbird_sparse_attention(q, k, v)``, commented out at
    kernels/cuda/src/torch_wrappers/ops.py:34-62): BigBird attention with the
    reference's block rule (global blocks, a sliding window ending at the
    diagonal block, random blocks rotated per query head,
    bigbird_pattern.py:23-41, 533-583), causal, scale 1/sqrt(D). The layout
    defaults are the CPU-runnable configuration's (64, 2, 3, 2). q/k/v as in
    sparse_attn (k/v may have fewer heads: GQA). The CSR is compiled on the
    device per (T_q, T_k) and cached."""
    layout = (int(block_size), int(global_blocks), int(sliding_blocks), int(random_blocks))
    key = (q.size(1), q.size(2), k.size(2), layout, str(q.device))
    hit = _BIGBIRD_OP_CACHE.get(key)
    if hit is None:
        hit = compile_bigbird([layout], q.size(1), q.size(2), k.size(2), layout[0], device=q.device)
        _BIGBIRD_OP_CACHE[key] = hit
        while len(_BIGBIRD_OP_CACHE) > 16:
            _BIGBIRD_OP_CACHE.pop(next(iter(_BIGBIRD_OP_CACHE)))
    return sparse_attn(q, k, v, hit[0], hit[1], layout[0])


_BIGBIRD_OP_CACHE: dict = {}


def _op_bigbird(layouts, n_heads, T_q, T_k, bs, variant, like):
    lay = [tuple(layouts[i:i + 4]) for i in range(0, len(layouts), 4)]
    return compile_bigbird(lay, n_heads, T_q, T_k, bs, variant=variant, device=like.device)


_LIB.impl("sparse_attn", _op_sparse_attn, "CUDA")
_LIB.impl("prefill_fwd", _op_prefill, "CUDA")
_LIB.impl("decode_fwd", _op_decode, "CUDA")
_LIB.impl("cuda_bigbird_sparse_attention", cuda_bigbird_sparse_attention, "CUDA")
_LIB.impl("compile_block_bitmap", compile_block_bitmap, "CUDA")
_LIB.impl("compile_token_mask", compile_token_mask, "CUDA")
_LIB.impl("compile_kv_block_list", compile_kv_block_list, "CUDA")
_LIB.impl("compile_bigbird", _op_bigbird, "CUDA")

@torch.library.register_fake("cuda_sparse_attention::cuda_bigbird_sparse_attention", lib=_LIB)
def _fake_bigbird(q, k, v, block_size=64, global_blocks=2, sliding_blocks=3, random_blocks=2):  # noqa: ARG001
    torch._check(q.dim() == 4 and k.dim() == 4 and v.dim() == 4)
    torch._check(q.device == k.device and q.device == v.device)
    torch._check(q.dtype == k.dtype and q.dtype == v.dtype)
    torch._check(q.shape[0] == k.shape[0] == v.shape[0])
    torch._check(k.shape[2] == v.shape[2] and q.shape[3] == k.shape[3] == v.shape[3])
    return torch.empty_like(q)


for _name in ("sparse_attn", "prefill_fwd", "decode_fwd"):
    def _fake(q, k, v, p, o, bs, scale=None, n_split=None):  # noqa: ARG001
        return torch.empty_like(q)
    torch.library.register_fake(f"cuda_sparse_attention::{_name}", _fake, lib=_LIB)
