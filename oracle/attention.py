"""Host restatement of the reference's masked-dense attention (test oracle only).

``masked_sdpa`` follows MaskedSdpaBackend.forward
(sparse_attentions/attention/masked_sdpa.py:23-68) line for line, in fp32 on
the CPU. ``masked_sdpa_chunked`` computes the same thing per (b, h) and per
block of query rows so that BASELINE-sized inputs fit in host memory; it is
checked against the unchunked form in the tests. ``csr_attention`` is the
same computation with the mask taken from a block CSR the way the reference
Triton kernel reads it (universal_sparse_attn.py:111-135).
"""
from __future__ import annotations

import math

import numpy as np
import torch

from .patterns import token_mask_from_csr


def _causal_keep(T_q: int, T_k: int, device="cpu") -> torch.Tensor:
    # utils.py:6-12 builds triu(ones(T_k, T_k), 1) = forbidden; masked_sdpa.py:40-45
    # keeps the last row for decode (T_q == 1) and the whole square otherwise.
    c = torch.triu(torch.ones(T_k, T_k, dtype=torch.bool, device=device), diagonal=1)
    if T_q == 1:
        return ~c[-1:, :]
    return ~c


def masked_sdpa(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, mask: torch.Tensor | None,
                kind: str = "mask") -> torch.Tensor:
    """MaskedSdpaBackend.forward for kind in {"mask", "local", "dense"} (masked_sdpa.py:23-68).

    q [B,H,T_q,D], k/v [B,H,T_k,D] (GQA callers repeat K/V first, as the
    reference hook does with repeat_kv), mask [H,T_q,T_k] bool (True = keep).
    """
    q, k, v = q.float(), k.float(), v.float()
    if kind == "dense":
        return torch.nn.functional.scaled_dot_product_attention(q, k, v, is_causal=True)
    B, H, T_q, D = q.shape
    T_k = k.size(2)
    scale = 1.0 / math.sqrt(D)
    scores = torch.matmul(q, k.transpose(-2, -1)) * scale
    combined = mask.unsqueeze(0) & _causal_keep(T_q, T_k, mask.device).unsqueeze(0).unsqueeze(0)
    scores = scores.masked_fill(~combined, float("-inf"))
    attn = torch.softmax(scores, dim=-1)
    attn = torch.nan_to_num(attn, nan=0.0)
    return torch.matmul(attn, v)


def masked_sdpa_chunked(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, mask_fn, *,
                        row_chunk: int = 1024, heads=None) -> torch.Tensor:
    """Same arithmetic as ``masked_sdpa`` one (b, h, query-row chunk) at a time.

    ``mask_fn(h, r0, r1) -> [r1-r0, T_k] bool`` supplies the pattern mask rows
    (True = keep), already AND-ed with nothing; the causal rule is applied here
    exactly as masked_sdpa.py:40-47 does (bottom-right for T_q == 1, top-left
    square otherwise, which for T_q == T_k is the same thing).
    K/V may have fewer heads than Q (GQA): head h reads kv head h // (H/Hkv),
    which equals the reference's repeat_kv expansion.
    """
    B, H, T_q, D = q.shape
    Hkv, T_k = k.size(1), k.size(2)
    rep = H // Hkv
    scale = 1.0 / math.sqrt(D)
    out = torch.zeros(B, H, T_q, D, dtype=torch.float32)
    hs = range(H) if heads is None else heads
    kpos = torch.arange(T_k)
    for b in range(B):
        for h in hs:
            kf = k[b, h // rep].float()
            vf = v[b, h // rep].float()
            for r0 in range(0, T_q, row_chunk):
                r1 = min(T_q, r0 + row_chunk)
                s = (q[b, h, r0:r1].float() @ kf.T) * scale
                if T_q == 1:
                    causal = torch.ones(1, T_k, dtype=torch.bool)
                else:
                    causal = kpos.unsqueeze(0) <= torch.arange(r0, r1).unsqueeze(1)
                keep = mask_fn(h, r0, r1) & causal
                s = s.masked_fill(~keep, float("-inf"))
                a = torch.nan_to_num(torch.softmax(s, dim=-1), nan=0.0)
                out[b, h, r0:r1] = a @ vf
    return out


def csr_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, pairs: np.ndarray,
                  offsets: np.ndarray, bs: int, *, row_chunk: int = 1024, heads=None) -> torch.Tensor:
    """fp32 attention restricted to the blocks of a CSR schedule, causal
    bottom-right and bounds masked (what universal_sparse_attn computes,
    universal_sparse_attn.py:111-153, in exact arithmetic)."""
    B, H, T_q, D = q.shape
    T_k = k.size(2)
    Hkv = k.size(1)
    rep = H // Hkv
    scale = 1.0 / math.sqrt(D)
    nqb = offsets.shape[1] - 1
    out = torch.zeros(B, H, T_q, D, dtype=torch.float32)
    hs = range(H) if heads is None else heads
    kpos = torch.arange(T_k)
    qoff = T_k - T_q
    for h in hs:
        allowed = torch.zeros(nqb, T_k, dtype=torch.bool)
        for qb in range(nqb):
            for kb in pairs[h, offsets[h, qb]:offsets[h, qb + 1]]:
                kb = int(kb)
                if kb >= 0:
                    allowed[qb, kb * bs:min(T_k, (kb + 1) * bs)] = True
        for b in range(B):
            kf = k[b, h // rep].float()
            vf = v[b, h // rep].float()
            for r0 in range(0, T_q, row_chunk):
                r1 = min(T_q, r0 + row_chunk)
                rows = torch.arange(r0, r1)
                keep = allowed[rows // bs] & (kpos.unsqueeze(0) <= (rows + qoff).unsqueeze(1))
                s = (q[b, h, r0:r1].float() @ kf.T) * scale
                s = s.masked_fill(~keep, float("-inf"))
                a = torch.nan_to_num(torch.softmax(s, dim=-1), nan=0.0)
                out[b, h, r0:r1] = a @ vf
    return out



def topk_sdpa(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, top_k: int) -> torch.Tensor:
    """MaskedSdpaBackend.forward for kind "topk" (masked_sdpa.py:51-63): causal
    mask first (last row for decode), then torch.topk of each score row, softmax
    over the kept entries, times V. q [B,H,T_q,D]; k/v with H heads (repeated)."""
    q, k, v = q.float(), k.float(), v.float()
    D = q.size(-1)
    T_q, T_k = q.size(2), k.size(2)
    top = min(top_k, T_k)
    scores = torch.matmul(q, k.transpose(-2, -1)) * (1.0 / math.sqrt(D))
    scores = scores.masked_fill(~_causal_keep(T_q, T_k).unsqueeze(0).unsqueeze(0), float("-inf"))
    vals, idx = torch.topk(scores, k=top, dim=-1)
    sparse = torch.full_like(scores, float("-inf")).scatter_(-1, idx, vals)
    attn = torch.nan_to_num(torch.softmax(sparse, dim=-1), nan=0.0)
    return torch.matmul(attn, v)

__all__ = ["masked_sdpa", "masked_sdpa_chunked", "csr_attention", "topk_sdpa", "token_mask_from_csr"]
