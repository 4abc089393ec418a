"""Backend layer: the reference's AttentionBackend API served by the sm_100a kernels.

``CudaSm100Backend`` is a drop-in for TritonUniversalBackend
(sparse_attentions/attention/triton_universal_backend.py:24-103): same
``forward(q, k, v, pattern) -> out`` and ``actual_backend`` property
(sparse_attentions/attention/base.py:9-40), registered by name the way
``_REGISTRY`` / ``get_backend`` do (sparse_attentions/attention/__init__.py:8-21).

Unlike the reference there is no silent fallback: unsupported inputs raise,
and ``actual_backend`` is always "cuda_sm100".
"""
from __future__ import annotations

import math
import weakref
from abc import ABC, abstractmethod

import torch

from . import ops as _ops
from .patterns import PatternMetadata


class AttentionBackend(ABC):
    """sparse_attentions/attention/base.py:9-40."""

    @abstractmethod
    def forward(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, pattern: PatternMetadata) -> torch.Tensor:
        ...

    @property
    def actual_backend(self) -> str:
        return type(self).__name__


class CudaSm100Backend(AttentionBackend):
    """Block-sparse attention on B200: tcgen05/TMEM prefill, split-KV decode.

    Accepts q [B,H,T_q,D] and k/v with H or H/G heads (GQA without repeat_kv).
    ``pattern.kind``:
      * "mask" / "local" with a CSR (block_pairs, block_pair_offsets, block_size);
        a pattern that only carries a token mask and a block_size is compiled
        on the device first (build_block_pairs_from_mask semantics);
      * "dense": full causal attention through a dense causal CSR (block 128) —
        bottom-right aligned, so decode is correct (unlike dense_sdpa.py:24);
      * "topk": data-dependent top-k per query row (``ops.topk_attention``:
        fp32 score GEMM, then masking, selection, softmax and PV in one kernel).
    """

    name = "cuda_sm100"

    def __init__(self, dense_block_size: int = 128):
        self.dense_block_size = dense_block_size
        self._dense_cache: dict = {}
        self._mask_cache: dict = {}
        self._validated: dict = {}
        self._last = "cuda_sm100"

    @property
    def actual_backend(self) -> str:
        return self._last

    def _dense_csr(self, H: int, T_q: int, T_k: int, device) -> tuple[torch.Tensor, torch.Tensor, int]:
        bs = self.dense_block_size
        key = (H, T_q, T_k, str(device))
        if key not in self._dense_cache:
            nkb = math.ceil(T_k / bs)
            nqb = math.ceil(T_q / bs)
            qoff = (T_k - T_q) // bs
            width = sum(min(qoff + q + 1, nkb) for q in range(nqb))  # exact nnz: no device read
            pairs, offsets = _ops.compile_bigbird([(bs, 0, nkb, 0)], H, T_q, T_k, bs, device=device, width=width)
            self._dense_cache[key] = (pairs, offsets, bs)
            while len(self._dense_cache) > 16:  # one entry per decode length: keep the recent ones
                self._dense_cache.pop(next(iter(self._dense_cache)))
        return self._dense_cache[key]

    def _validate(self, pairs, offsets, T_q: int, T_k: int, bs: int) -> None:
        """A CSR from outside this package (e.g. the reference's own pattern
        objects) is validated once per tensor pair and contents (sa_validate_csr;
        the tensors are held by weak reference, their in-place version counters
        detect changes); a violation raises SaError (SA_ERR_CSR)."""
        key = (id(pairs), id(offsets), T_q, T_k, bs)
        hit = self._validated.get(key)
        if hit is not None and hit[0]() is pairs and hit[1]() is offsets and \
                hit[2] == (pairs._version, offsets._version):
            return
        _ops.validate_csr(pairs, offsets, T_q, T_k, bs)
        self._validated[key] = (weakref.ref(pairs), weakref.ref(offsets), (pairs._version, offsets._version))
        while len(self._validated) > 64:
            self._validated.pop(next(iter(self._validated)))

    def forward(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, pattern: PatternMetadata) -> torch.Tensor:
        if not q.is_cuda:
            raise RuntimeError("cuda_sm100 backend needs CUDA tensors (no CPU fallback)")
        H, T_q, T_k = q.size(1), q.size(2), k.size(2)
        if pattern.kind == "dense":
            pairs, offsets, bs = self._dense_csr(H, T_q, T_k, q.device)
        elif pattern.kind in ("mask", "local"):
            pairs, offsets, bs = pattern.block_pairs, pattern.block_pair_offsets, pattern.block_size
            if pairs is None or offsets is None:
                if pattern.mask is None or bs is None:
                    raise ValueError("cuda_sm100 needs a block CSR (block_pairs/block_pair_offsets/block_size) "
                                     "or a token mask plus block_size")
                key = (id(pattern.mask), bs)
                if key not in self._mask_cache:
                    self._mask_cache = {key: _ops.compile_token_mask(pattern.mask, bs)}
                pairs, offsets = self._mask_cache[key]
            if bs is None:
                raise ValueError("pattern.block_size is None")
            if not getattr(pattern, "_sa_compiled", False) and pattern.block_pairs is not None:
                self._validate(pairs, offsets, T_q, T_k, int(bs))
        elif pattern.kind == "topk":
            self._last = "cuda_sm100"
            return _ops.topk_attention(q, k, v, int(pattern.topk))
        else:
            raise NotImplementedError(f"cuda_sm100 does not implement pattern kind {pattern.kind!r}")
        self._last = "cuda_sm100"
        return _ops.sparse_attn(q, k, v, pairs, offsets, int(bs))


_REGISTRY: dict[str, type[AttentionBackend]] = {"cuda_sm100": CudaSm100Backend}


def get_backend(name: str, **kwargs) -> AttentionBackend:
    """sparse_attentions/attention/__init__.py:17-21."""
    if name not in _REGISTRY:
        raise ValueError(f"Unknown backend {name!r}. Available: {', '.join(sorted(_REGISTRY))}")
    return _REGISTRY[name](**kwargs)


def register_with_reference(registry: dict | None = None) -> dict:
    """Insert "cuda_sm100" into the reference's backend registry.

    With ``registry=None`` the registry of an importable
    ``sparse_attentions.attention`` package is used (that package must be on
    sys.path); its ``get_backend("cuda_sm100")`` then returns this backend.
    """
    if registry is None:
        from sparse_attentions import attention as ref_attention  # type: ignore
        registry = ref_attention._REGISTRY
    registry["cuda_sm100"] = CudaSm100Backend
    return registry
