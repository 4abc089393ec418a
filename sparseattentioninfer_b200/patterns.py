"""Pattern layer: the reference's pattern API with the CSR compiled on the device.

Mirrors sparse_attentions/patterns/{base,bigbird_pattern,local_window,
causal_dense,topk_pattern}.py: same class names, constructor arguments,
``build(q, k, causal=True) -> PatternMetadata`` and PatternMetadata fields.
Differences, all deliberate:

* ``block_pairs`` / ``block_pair_offsets`` come from the CUDA pattern compiler
  (bit-exact with the reference's Python loops, see sa_pattern.cu);
* the O(H*T^2) token ``mask`` is not built unless ``materialize_mask=True``
  (the CUDA backend never reads it; masked-dense interop can ask for it);
* ``kv_block_list`` (legacy padded schedule) is built only on request;
* BigBird layouts can be given explicitly (``layouts=``), the supported form
  of the reference's ``_layout_cache`` injection;
* decode builds (T_q == 1) take a no-sync path whose block_pairs width is the
  layout bound g+w+r instead of the exact max nnz (``exact_width=False``).
"""
from __future__ import annotations

import math
from abc import ABC, abstractmethod
from dataclasses import dataclass
from typing import Sequence

import torch

from . import _capi
from . import ops as _ops


@dataclass
class PatternMetadata:
    """Same fields as sparse_attentions/patterns/base.py:11-33."""

    kind: str
    mask: torch.Tensor | None = None
    topk: int | None = None
    keep_ratio: float = 1.0
    build_time_ms: float = 0.0
    block_size: int | None = None
    kv_block_list: torch.Tensor | None = None
    block_pairs: torch.Tensor | None = None
    block_pair_offsets: torch.Tensor | None = None


def _compiled(md: PatternMetadata) -> PatternMetadata:
    """Marks a CSR produced by this package's device compiler: the backend skips
    its one-time validation (sa_validate_csr) for such metadata."""
    md._sa_compiled = True
    return md


class SparsePattern(ABC):
    """sparse_attentions/patterns/base.py:136-154."""

    @abstractmethod
    def build(self, q: torch.Tensor, k: torch.Tensor, causal: bool = True) -> PatternMetadata: ...


def next_pow2_min16(x: int) -> int:
    """bigbird_pattern.py:97-103."""
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
    w = min(2, budget)
    return bs, 1, w, max(0, budget - 1 - w)


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
    bs = max(1, min(seq_len, int(math.sqrt(max(1, target))) if block_size is None else int(block_size)))
    nb = math.ceil(seq_len / bs)
    budget = max(1, min(nb, math.ceil(target / bs)))
    w = min(2, budget)
    return bs, 1, w, max(0, budget - 1 - w)


def causal_block_keep_ratio(nnz_total: int, H: int, nqb: int, T_q: int, T_k: int, bs: int) -> float:
    """_causal_block_keep_ratio_from_offsets (bigbird_pattern.py:106-125), from the
    total nnz instead of a host copy of the offsets."""
    nkb = math.ceil(T_k / bs)
    qoff = max(0, T_k - T_q) // bs
    total = sum(min(qoff + q + 1, nkb) for q in range(nqb))
    if total <= 0:
        return 0.0
    return min(1.0, nnz_total / (H * total))


def _device_key(device: torch.device) -> str:
    return f"{device.type}:{device.index}"


def _token_mask_from_csr(pairs: torch.Tensor, offsets: torch.Tensor, bs: int, T_q: int, T_k: int,
                         force_diag: bool) -> torch.Tensor:
    """Device token mask of a CSR: block in row & causal (bottom-right); with
    force_diag the query->own-position entry is True (bigbird_pattern.py:527-529)."""
    H, nq1 = offsets.shape
    nqb = nq1 - 1
    nkb = max(math.ceil(T_k / bs), int(pairs.max().item()) + 1)
    dev = pairs.device
    counts = (offsets[:, 1:] - offsets[:, :-1]).long()
    rows = torch.repeat_interleave(torch.arange(H * nqb, device=dev), counts.reshape(-1))
    starts = offsets[:, :-1].long() + torch.arange(H, device=dev).view(-1, 1) * pairs.size(1)
    idx = torch.repeat_interleave(starts.reshape(-1), counts.reshape(-1))
    pos = torch.arange(idx.numel(), device=dev) - torch.repeat_interleave(
        torch.cumsum(counts.reshape(-1), 0) - counts.reshape(-1), counts.reshape(-1))
    kb = pairs.reshape(-1)[idx + pos].long()
    bm = torch.zeros(H * nqb, nkb, dtype=torch.bool, device=dev)
    bm[rows, kb] = True
    bm = bm.view(H, nqb, nkb)
    q2b = torch.arange(T_q, device=dev) // bs
    k2b = torch.arange(T_k, device=dev) // bs
    m = bm[:, q2b][:, :, k2b]
    qpos = (T_k - T_q) + torch.arange(T_q, device=dev)
    m &= (torch.arange(T_k, device=dev).unsqueeze(0) <= qpos.unsqueeze(1)).unsqueeze(0)
    if force_diag:
        m[:, torch.arange(T_q, device=dev), qpos] = True
    return m


class _BigBirdBase(SparsePattern):
    variant = _capi.SA_BIGBIRD

    def __init__(self, n_heads: int, *, materialize_mask: bool = False, build_kv_block_list: bool = False,
                 exact_width: bool | None = None):
        self.n_heads = n_heads
        self.materialize_mask = materialize_mask
        self.build_kv_block_list = build_kv_block_list
        self.exact_width = exact_width
        self._csr_cache: dict = {}
        self.last_layout = None
        self.last_group_layouts = None

    def _layouts(self, T_q: int, T_k: int) -> tuple[tuple[int, int, int, int], ...]:
        raise NotImplementedError

    def _width_bound(self, layouts, T_q: int, T_k: int, bs: int) -> int:
        nqb = math.ceil(T_q / bs)
        nkb = math.ceil(T_k / bs)
        per_row = max(g + w + r for _, g, w, r in layouts)
        if self.variant == _capi.SA_BIGBIRD2:
            return (nqb - 1) * per_row + max(nkb, per_row)
        return nqb * per_row

    def build(self, q: torch.Tensor, k: torch.Tensor, causal: bool = True) -> PatternMetadata:
        T_q, T_k = q.size(2), k.size(2)
        device = q.device
        layouts = self._layouts(T_q, T_k)
        self.last_group_layouts = layouts
        self.last_layout = layouts[0] if len(layouts) == 1 else None
        bs = next_pow2_min16(layouts[0][0])
        # A decode row depends on T_k only through its block (T_k-1)//bs and the
        # block count ceil(T_k/bs): decoding reuses one build for a whole block.
        tk_key = ((T_k - 1) // bs, -(-T_k // bs)) if T_q == 1 else T_k
        key = (T_q, tk_key, _device_key(device), layouts)
        if key not in self._csr_cache:
            exact = self.exact_width if self.exact_width is not None else T_q > 1
            width = None if exact else self._width_bound(layouts, T_q, T_k, bs)
            pairs, offsets = _ops.compile_bigbird(layouts, self.n_heads, T_q, T_k, bs, variant=self.variant,
                                                  device=device, width=width)
            if exact:
                nnz = int(offsets[:, -1].sum().item())
                keep = causal_block_keep_ratio(nnz, self.n_heads, offsets.size(1) - 1, T_q, T_k, bs)
            else:
                keep = float("nan")  # computed lazily by keep_ratio_of() to stay sync-free
            self._csr_cache[key] = (pairs, offsets, keep)
            while len(self._csr_cache) > 16:  # decode builds one entry per T_k: keep the recent ones
                self._csr_cache.pop(next(iter(self._csr_cache)))
        pairs, offsets, keep = self._csr_cache[key]
        mask = None
        if self.materialize_mask:
            mask = _token_mask_from_csr(pairs, offsets, bs, T_q, T_k, force_diag=True)
        kvl = None
        if self.build_kv_block_list:
            kvl = self._kv_block_list(pairs, offsets, layouts, T_q, T_k, bs)
        return _compiled(PatternMetadata(kind="mask", mask=mask, keep_ratio=keep, block_size=bs, kv_block_list=kvl,
                                         block_pairs=pairs, block_pair_offsets=offsets))

    def _kv_block_list(self, pairs, offsets, layouts, T_q, T_k, bs):
        """Legacy padded schedule (bigbird_pattern.py:585-634) from the CSR rows."""
        max_kv = max(1, max(g + w + r for _, g, w, r in layouts))
        if self.variant == _capi.SA_BIGBIRD2:
            max_kv = max(math.ceil(T_k / bs), max_kv)
        H, nq1 = offsets.shape
        nqb = nq1 - 1
        counts = (offsets[:, 1:] - offsets[:, :-1]).long()
        slot = torch.arange(max_kv, device=pairs.device).view(1, 1, -1)
        gidx = (offsets[:, :-1].long().unsqueeze(-1) + slot).clamp(max=pairs.size(1) - 1)
        vals = torch.gather(pairs.long(), 1, gidx.view(H, -1)).view(H, nqb, max_kv)
        return torch.where(slot < counts.unsqueeze(-1), vals, torch.full_like(vals, -1)).to(torch.int32)


class BigBirdPattern(_BigBirdBase):
    """bigbird_pattern.py:130-335: layout from top_k (bigbird_layout_from_topk)."""

    def __init__(self, top_k: int, n_heads: int, **kw):
        super().__init__(n_heads, **kw)
        self.top_k = top_k

    def _layouts(self, T_q, T_k):
        return (bigbird_layout_from_topk(T_k, self.top_k),)


class BigBird2Pattern(BigBirdPattern):
    """bigbird_pattern.py:639-806: the last query-block row attends to every key block."""

    variant = _capi.SA_BIGBIRD2


class BigBirdKeepRatioPattern(_BigBirdBase):
    """bigbird_pattern.py:366-634: one keep ratio, or one sparsity per KV group.

    ``layouts=`` fixes the (bs, g, w, r) per group for every shape (what the
    reference reaches by writing ``_layout_cache``); ``_layout_cache`` itself is
    honoured too."""

    def __init__(self, *, keep_ratio: float | None = None, group_sparsities: Sequence[float] | None = None,
                 n_heads: int, n_kv_heads: int | None = None,
                 layouts: Sequence[Sequence[int]] | None = None, **kw):
        super().__init__(n_heads, **kw)
        if layouts is None and keep_ratio is None and group_sparsities is None:
            raise ValueError("Either keep_ratio or group_sparsities must be provided.")
        if keep_ratio is not None and group_sparsities is not None:
            raise ValueError("Provide keep_ratio or group_sparsities, not both.")
        self.keep_ratio = keep_ratio
        self.group_sparsities = None if group_sparsities is None else tuple(float(x) for x in group_sparsities)
        self.fixed_layouts = None if layouts is None else tuple(tuple(int(v) for v in l) for l in layouts)
        if self.group_sparsities is not None:
            if n_kv_heads is not None and len(self.group_sparsities) != n_kv_heads:
                raise ValueError(f"group_sparsities has length {len(self.group_sparsities)}, "
                                 f"but n_kv_heads is {n_kv_heads}.")
            if any(not 0.0 <= x < 1.0 for x in self.group_sparsities):
                raise ValueError("All group sparsities must satisfy 0 <= sparsity < 1.")
            self.group_keep_ratios = tuple(1.0 - x for x in self.group_sparsities)
        elif keep_ratio is not None:
            self.group_keep_ratios = (float(keep_ratio),)
        else:
            self.group_keep_ratios = tuple(1.0 for _ in self.fixed_layouts)
        self.group_count = len(self.fixed_layouts) if self.fixed_layouts else len(self.group_keep_ratios)
        if n_heads % self.group_count:
            raise ValueError(f"n_heads={n_heads} must be divisible by group_count={self.group_count}.")
        self.group_size = n_heads // self.group_count
        self._layout_cache: dict = {}

    def _layouts(self, T_q, T_k):
        key = (T_q, T_k)
        if key in self._layout_cache:
            return tuple(tuple(x) for x in self._layout_cache[key])
        if self.fixed_layouts is not None:
            return self.fixed_layouts
        decode = T_q != T_k
        if len(self.group_keep_ratios) == 1:
            lay = (bigbird_layout_from_keep_ratio(T_k, self.group_keep_ratios[0], decode=decode),)
        else:
            desired = [bigbird_layout_from_keep_ratio(T_k, kr, decode=decode)[0] for kr in self.group_keep_ratios]
            shared = next_pow2_min16(min(desired))
            lay = tuple(bigbird_layout_from_keep_ratio(T_k, kr, decode=decode, block_size=shared)
                        for kr in self.group_keep_ratios)
        self._layout_cache[key] = lay
        return lay


class BlockMaskPattern(SparsePattern):
    """Arbitrary retained-QK^T block mask: a block bitmap [H, NQB, NKB] (or a
    callable (T_q, T_k) -> bitmap) compiled on the device. The reference route
    for this is a token mask through build_block_pairs_from_mask (base.py:36-89)."""

    def __init__(self, bitmap, block_size: int, *, materialize_mask: bool = False):
        self.bitmap = bitmap
        self.block_size = block_size
        self.materialize_mask = materialize_mask
        self._cache: dict = {}

    def build(self, q, k, causal: bool = True) -> PatternMetadata:
        T_q, T_k = q.size(2), k.size(2)
        key = (T_q, T_k, _device_key(q.device))
        if key not in self._cache:
            bm = self.bitmap(T_q, T_k) if callable(self.bitmap) else self.bitmap
            bm = torch.as_tensor(bm).to(device=q.device, dtype=torch.uint8)
            pairs, offsets = _ops.compile_block_bitmap(bm)
            nnz = int(offsets[:, -1].sum().item())
            keep = causal_block_keep_ratio(nnz, offsets.size(0), offsets.size(1) - 1, T_q, T_k, self.block_size)
            self._cache[key] = (pairs, offsets, keep)
        pairs, offsets, keep = self._cache[key]
        mask = _token_mask_from_csr(pairs, offsets, self.block_size, T_q, T_k, False) if self.materialize_mask else None
        return _compiled(PatternMetadata(kind="mask", mask=mask, keep_ratio=keep, block_size=self.block_size,
                                         block_pairs=pairs, block_pair_offsets=offsets))


class LocalWindowPattern(SparsePattern):
    """local_window.py:11-80. The CSR (when block_size is given) is compiled on
    the device from the window's token mask, like build_block_pairs_from_mask."""

    def __init__(self, window_size: int, block_size: int | None = None, *, materialize_mask: bool = True):
        self.window_size = window_size
        self.block_size = block_size
        self.materialize_mask = materialize_mask
        self._cache: dict = {}

    def _mask(self, T_q, T_k, H, device, causal):
        W = self.window_size
        qoff = max(0, T_k - T_q)
        rows = (qoff + torch.arange(T_q, device=device)).unsqueeze(1)
        cols = torch.arange(T_k, device=device).unsqueeze(0)
        m = (cols >= rows - W + 1) & (cols <= rows)
        return m.unsqueeze(0).expand(H, -1, -1)

    def build(self, q, k, causal: bool = True) -> PatternMetadata:
        T_q, T_k, H = q.size(2), k.size(2), q.size(1)
        key = (T_q, T_k, H, _device_key(q.device), causal)
        if key not in self._cache:
            mask = self._mask(T_q, T_k, H, q.device, causal)
            pairs = offsets = None
            if self.block_size is not None:
                pairs, offsets = _ops.compile_token_mask(mask.contiguous(), self.block_size)
            self._cache[key] = (mask, pairs, offsets)
        mask, pairs, offsets = self._cache[key]
        W = self.window_size
        qoff = max(0, T_k - T_q)
        keep = min(1.0, sum(min(W, qoff + i + 1) for i in range(T_q)) / max(1, T_q * T_k))
        return _compiled(PatternMetadata(kind="local", mask=mask if self.materialize_mask else None,
                                         keep_ratio=keep, block_size=self.block_size, block_pairs=pairs,
                                         block_pair_offsets=offsets))


class DenseCausalPattern(SparsePattern):
    """causal_dense.py:7-11."""

    def build(self, q, k, causal: bool = True) -> PatternMetadata:
        return PatternMetadata(kind="dense", keep_ratio=1.0)


class TopKPattern(SparsePattern):
    """topk_pattern.py:44-62: data-dependent, the backend selects each query row's
    top_k causal scores (CudaSm100Backend: ops.topk_attention). keep_ratio as
    the reference computes it (:29-41)."""

    def __init__(self, top_k: int):
        self.top_k = top_k

    def build(self, q, k, causal: bool = True) -> PatternMetadata:
        T_q, T_k = q.size(2), k.size(2)
        top = min(self.top_k, T_k)
        if T_k <= 0:
            keep = 0.0
        elif T_q == T_k:
            keep = min(1.0, sum(min(top, pos + 1) for pos in range(T_k)) / max(1, T_k * (T_k + 1) // 2))
        else:
            keep = min(top, T_k) / T_k
        return PatternMetadata(kind="topk", topk=self.top_k, keep_ratio=keep)


__all__ = [
    "PatternMetadata", "SparsePattern", "BigBirdPattern", "BigBird2Pattern", "BigBirdKeepRatioPattern",
    "BlockMaskPattern", "LocalWindowPattern", "DenseCausalPattern", "TopKPattern",
    "bigbird_layout_from_topk", "bigbird_layout_from_keep_ratio", "next_pow2_min16",
]
