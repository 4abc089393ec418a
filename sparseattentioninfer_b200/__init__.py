"""B200-native block-sparse attention backend (sm_100a, tcgen05/TMEM/TMA).

Drop-in for the pattern/backend abstraction of rrroooyyywang/SparseAttentionInfer:

    from sparseattentioninfer_b200 import BigBirdKeepRatioPattern, get_backend
    pattern = BigBirdKeepRatioPattern(keep_ratio=0.2, n_heads=32)
    out = get_backend("cuda_sm100").forward(q, k, v, pattern.build(q, k))

Importing the package loads the in-tree CUDA library ``_lib/libsa_b200.so``
and raises ImportError if it is missing: there is no CPU fallback.
"""
from . import _capi

_capi.load()

from . import ops  # noqa: E402  (registers torch.ops.cuda_sparse_attention.*)
from .backend import AttentionBackend, CudaSm100Backend, get_backend, register_with_reference  # noqa: E402
from .patterns import (  # noqa: E402
    BigBird2Pattern,
    BigBirdKeepRatioPattern,
    BigBirdPattern,
    BlockMaskPattern,
    DenseCausalPattern,
    LocalWindowPattern,
    PatternMetadata,
    SparsePattern,
    TopKPattern,
)

__version__ = "0.1.0"

__all__ = [
    "AttentionBackend", "CudaSm100Backend", "get_backend", "register_with_reference", "ops",
    "PatternMetadata", "SparsePattern", "BigBirdPattern", "BigBird2Pattern", "BigBirdKeepRatioPattern",
    "BlockMaskPattern", "LocalWindowPattern", "DenseCausalPattern", "TopKPattern",
]
