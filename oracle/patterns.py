"""Host restatement of the reference's pattern builders (test oracle only).

Each function cites the reference file:line it restates. Pure Python / numpy
loops: fine for the sizes the parity tests use (and for full BASELINE sizes,
where the reference itself runs the same loops).
"""
from __future__ import annotations

import math
from typing import Sequence

import numpy as np
import torch


def next_pow2_min16(x: int) -> int:
    """bigbird_pattern.py:97-103 (_next_pow2_min16)."""
    p = max(16, x)
    r = 1
    while r < p:
        r <<= 1
    return r


def bigbird_layout_from_topk(seq_len: int, top_k: int) -> tuple[int, int, int, int]:
    """bigbird_pattern.py:12-20."""
    if seq_len <= 1:
        return 1, 1, 1, 0
    bs = max(1, min(seq_len, int(math.sqrt(max(1, top_k)))))
    budget = max(1, math.ceil(top_k / bs))
    g = 1
    w = min(2, budget)
    r = max(0, budget - g - w)
    return bs, g, w, r


def bigbird_layout_from_keep_ratio(seq_len: int, keep_ratio: float, *, decode: bool,
                                   block_size: int | None = None) -> tuple[int, int, int, int]:
    """bigbird_pattern.py:338-363."""
    if seq_len <= 1:
        return 1, 1, 1, 0
    keep_ratio = min(max(keep_ratio, 1.0 / seq_len), 1.0)
    if decode:
        target = max(1, math.ceil(keep_ratio * seq_len))
    else:
        target = max(1, math.ceil(keep_ratio * ((seq_len + 1) / 2)))
    if block_size is None:
        bs = max(1, min(seq_len, int(math.sqrt(max(1, target)))))
    else:
        bs = max(1, min(seq_len, int(block_size)))
    nb = math.ceil(seq_len / bs)
    budget = max(1, min(nb, math.ceil(target / bs)))
    g = 1
    w = min(2, budget)
    r = max(0, budget - g - w)
    return bs, g, w, r


def select_bigbird_random_block_ids(query_block: int, head_idx: int, num_blocks: int,
                                    global_blocks: int, sliding_blocks: int,
                                    random_blocks: int) -> list[int]:
    """bigbird_pattern.py:23-41: deterministic rotation, not a RNG."""
    if random_blocks <= 0 or query_block <= 0:
        return []
    local_start = max(global_blocks, query_block - sliding_blocks + 1)
    cands = [b for b in range(global_blocks, query_block) if b < local_start]
    if not cands:
        return []
    if len(cands) <= random_blocks:
        return cands
    off = (head_idx * 131 + query_block * 17 + num_blocks * 7) % len(cands)
    rot = cands[off:] + cands[:off]
    return rot[:random_blocks]


def _row_set(qb_abs: int, h: int, nkb: int, g: int, w: int, r: int) -> set[int]:
    allowed = set(range(g))
    ls = max(0, qb_abs - w + 1)
    allowed.update(range(ls, min(qb_abs + 1, nkb)))
    allowed.update(select_bigbird_random_block_ids(qb_abs, h, nkb, g, w, r))
    return allowed


def bigbird_csr(layouts: Sequence[tuple[int, int, int, int]], n_heads: int, T_q: int, T_k: int,
                *, block_size: int | None = None, variant: str = "bigbird") -> tuple[np.ndarray, np.ndarray]:
    """CSR of BigBirdKeepRatioPattern._get_block_pairs (bigbird_pattern.py:533-583);
    with one layout also BigBirdPattern._get_block_pairs (:212-271); variant
    "bigbird2" is BigBird2Pattern._get_block_pairs (:697-753).

    Head h uses layouts[h // (n_heads // len(layouts))]. The block size is
    ``block_size`` or _next_pow2_min16(layouts[0][0]) (:545).
    Returns (pairs [H, max(1, max_nnz)] int32 zero padded, offsets [H, NQB+1]).
    """
    bs = block_size if block_size is not None else next_pow2_min16(layouts[0][0])
    nqb = math.ceil(T_q / bs)
    nkb = math.ceil(T_k / bs)
    qoff = max(0, T_k - T_q) // bs
    hpg = n_heads // len(layouts)
    rows: list[list[int]] = []
    offs: list[list[int]] = []
    for h in range(n_heads):
        _, g, w, r = layouts[h // hpg]
        o = [0]
        pr: list[int] = []
        for ql in range(nqb):
            qa = qoff + ql
            if variant == "bigbird2" and ql == nqb - 1:
                allowed = set(range(nkb))
            else:
                allowed = _row_set(qa, h, nkb, g, w, r)
            pr.extend(sorted(allowed))
            o.append(len(pr))
        rows.append(pr)
        offs.append(o)
    mp = max(1, max(len(x) for x in rows))
    pairs = np.zeros((n_heads, mp), dtype=np.int32)
    for h, pr in enumerate(rows):
        pairs[h, : len(pr)] = pr
    return pairs, np.asarray(offs, dtype=np.int32)


def bigbird_kv_block_list(layouts, n_heads, T_q, T_k, *, variant: str = "bigbird") -> np.ndarray:
    """Legacy padded schedule, bigbird_pattern.py:585-634 (and :273-335, :755-806)."""
    bs = next_pow2_min16(layouts[0][0])
    nqb = math.ceil(T_q / bs)
    nkb = math.ceil(T_k / bs)
    qoff = max(0, T_k - T_q) // bs
    hpg = n_heads // len(layouts)
    max_kv = max(1, max(g + w + r for _, g, w, r in layouts))
    if variant == "bigbird2":
        max_kv = max(nkb, max_kv)
    out = np.full((n_heads, nqb, max_kv), -1, dtype=np.int32)
    for h in range(n_heads):
        _, g, w, r = layouts[h // hpg]
        for ql in range(nqb):
            qa = qoff + ql
            if variant == "bigbird2" and ql == nqb - 1:
                allowed = set(range(nkb))
            else:
                allowed = _row_set(qa, h, nkb, g, w, r)
            for slot, kb in enumerate(sorted(allowed)[:max_kv]):
                out[h, ql, slot] = kb
    return out


def causal_block_keep_ratio(offsets: np.ndarray, T_q: int, T_k: int, bs: int) -> float:
    """_causal_block_keep_ratio_from_offsets, bigbird_pattern.py:106-125."""
    H = offsets.shape[0]
    nqb = offsets.shape[1] - 1
    nkb = math.ceil(T_k / bs)
    qoff = max(0, T_k - T_q) // bs
    total = sum(min(qoff + q + 1, nkb) for q in range(nqb))
    if total <= 0:
        return 0.0
    kept = int(offsets[:, -1].astype(np.int64).sum())
    return min(1.0, kept / (H * total))


def bigbird_token_mask(layouts, n_heads: int, T_q: int, T_k: int, *, variant: str = "bigbird") -> torch.Tensor:
    """Token mask of BigBirdKeepRatioPattern._get_mask (bigbird_pattern.py:487-531):
    block mask at the layout's own block size, AND causal (bottom-right), with
    the diagonal query->own-position forced True. For variant "bigbird2",
    BigBird2Pattern._get_mask (:646-695)."""
    qoff = max(0, T_k - T_q)
    qpos = qoff + torch.arange(T_q)
    kpos = torch.arange(T_k)
    causal = kpos.unsqueeze(0) <= qpos.unsqueeze(1)
    hpg = n_heads // len(layouts)
    out = torch.zeros(n_heads, T_q, T_k, dtype=torch.bool)
    for h in range(n_heads):
        bs, g, w, r = layouts[h // hpg]
        nkb = math.ceil(T_k / bs)
        nqb = math.ceil(T_q / bs)
        qbo = qoff // bs
        bm = torch.zeros(nqb, nkb, dtype=torch.bool)
        for ql in range(nqb):
            qa = qbo + ql
            if variant == "bigbird2" and ql == nqb - 1:
                bm[ql, :] = True
                continue
            bm[ql, :g] = True
            ls = max(0, qa - w + 1)
            bm[ql, ls:min(qa + 1, nkb)] = True
            ids = select_bigbird_random_block_ids(qa, h, nkb, g, w, r)
            if ids:
                bm[ql, torch.tensor(ids)] = True
        q2b = torch.arange(T_q) // bs
        k2b = torch.arange(T_k) // bs
        out[h] = bm[q2b][:, k2b] & causal
    out[:, torch.arange(T_q), qpos] = True
    return out


def local_window_token_mask(window: int, H: int, T_q: int, T_k: int) -> torch.Tensor:
    """LocalWindowPattern._build_mask (local_window.py:62-72)."""
    qoff = max(0, T_k - T_q)
    rows = (qoff + torch.arange(T_q)).unsqueeze(1)
    cols = torch.arange(T_k).unsqueeze(0)
    m = (cols >= rows - window + 1) & (cols <= rows)
    return m.unsqueeze(0).expand(H, -1, -1).clone()


def block_bitmap_from_token_mask(mask: torch.Tensor, bs: int) -> np.ndarray:
    """Block coarsening of build_block_pairs_from_mask (patterns/base.py:58-73)."""
    H, T_q, T_k = mask.shape
    nqb, nkb = math.ceil(T_q / bs), math.ceil(T_k / bs)
    m = torch.zeros(H, nqb * bs, nkb * bs, dtype=torch.bool)
    m[:, :T_q, :T_k] = mask
    return m.reshape(H, nqb, bs, nkb, bs).any(dim=4).any(dim=2).numpy().astype(np.uint8)


def csr_from_block_bitmap(bitmap: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """CSR loop of build_block_pairs_from_mask (patterns/base.py:75-89)."""
    H, nqb, _ = bitmap.shape
    rows, offs = [], []
    for h in range(H):
        o = [0]
        pr: list[int] = []
        for q in range(nqb):
            pr.extend(np.nonzero(bitmap[h, q])[0].tolist())
            o.append(len(pr))
        rows.append(pr)
        offs.append(o)
    mp = max(1, max(len(x) for x in rows))
    pairs = np.zeros((H, mp), dtype=np.int32)
    for h, pr in enumerate(rows):
        pairs[h, : len(pr)] = pr
    return pairs, np.asarray(offs, dtype=np.int32)


def csr_from_kv_block_list(kvl: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """kv_block_list_to_pairs (patterns/base.py:92-133)."""
    H, nqb, _ = kvl.shape
    rows, offs = [], []
    for h in range(H):
        o = [0]
        pr: list[int] = []
        for q in range(nqb):
            row = kvl[h, q]
            pr.extend(int(x) for x in row[row >= 0])
            o.append(len(pr))
        rows.append(pr)
        offs.append(o)
    mp = max(1, max(len(x) for x in rows))
    pairs = np.zeros((H, mp), dtype=np.int32)
    for h, pr in enumerate(rows):
        pairs[h, : len(pr)] = pr
    return pairs, np.asarray(offs, dtype=np.int32)


def token_mask_from_csr(pairs: np.ndarray, offsets: np.ndarray, bs: int, T_q: int, T_k: int) -> torch.Tensor:
    """Token-level view of what the reference Triton kernel computes from a CSR
    (universal_sparse_attn.py:111-135): key j visible to query i iff block j//bs
    is in row (h, i//bs) and j <= i + (T_k - T_q) and j < T_k."""
    H = offsets.shape[0]
    nqb = offsets.shape[1] - 1
    nkb_all = max(int(pairs.max()) + 1 if pairs.size else 1, math.ceil(T_k / bs))
    bm = torch.zeros(H, nqb, nkb_all, dtype=torch.bool)
    for h in range(H):
        for q in range(nqb):
            for kb in pairs[h, offsets[h, q]:offsets[h, q + 1]]:
                if kb >= 0:
                    bm[h, q, int(kb)] = True
    q2b = torch.arange(T_q) // bs
    k2b = torch.arange(T_k) // bs
    m = bm[:, q2b][:, :, k2b]
    qpos = (T_k - T_q) + torch.arange(T_q)
    causal = torch.arange(T_k).unsqueeze(0) <= qpos.unsqueeze(1)
    return m & causal.unsqueeze(0)

