"""The drop-in against the real reference, where its checkout is present (the
build container; skipped elsewhere): registering this backend in the
reference's own registry (sparse_attentions/attention/__init__.py:8-21) makes
its get_backend("cuda_sm100") return CudaSm100Backend, next to the reference's
backends; and the ops fragment carries the reference's intended op name
(kernels/cuda/src/torch_wrappers/ops.py:34-62)."""
from __future__ import annotations

import os
import sys

import pytest
import torch

import sparseattentioninfer_b200 as sa

REF = os.environ.get("SA_REFERENCE_DIR", "/root/reference")
need_ref = pytest.mark.skipif(not os.path.isdir(os.path.join(REF, "sparse_attentions")),
                              reason="reference checkout not present")


@need_ref
def test_register_into_the_reference_registry():
    sys.path.insert(0, REF)
    try:
        from sparse_attentions import attention as ref_attention
        before = set(ref_attention._REGISTRY)
        sa.register_with_reference()
        be = ref_attention.get_backend("cuda_sm100")
        assert isinstance(be, sa.CudaSm100Backend)
        assert be.actual_backend == "cuda_sm100"
        assert before <= set(ref_attention._REGISTRY)            # the reference's own backends stay
        assert isinstance(ref_attention.get_backend("masked_sdpa"), ref_attention.MaskedSdpaBackend)
        with pytest.raises(ValueError, match="Unknown backend"):
            ref_attention.get_backend("no_such_backend")
    finally:
        sys.path.remove(REF)


@need_ref
def test_reference_pattern_metadata_is_accepted_as_is():
    """A PatternMetadata built by the reference's own BigBirdKeepRatioPattern is
    what the reference's callers hand to forward(): its fields are the ones this
    backend reads (the GPU test feeds such metadata through the kernel)."""
    sys.path.insert(0, REF)
    try:
        from sparse_attentions.patterns import BigBirdKeepRatioPattern
        pat = BigBirdKeepRatioPattern(keep_ratio=0.5, n_heads=4)
        pat._layout_cache[(256, 256)] = ((64, 2, 3, 2),)
        md = pat.build(torch.zeros(1, 4, 256, 8), torch.zeros(1, 4, 256, 8))
        for field in ("kind", "mask", "block_size", "block_pairs", "block_pair_offsets"):
            assert hasattr(md, field), field
        assert md.kind == "mask" and md.block_size == 64
        assert md.block_pairs.dtype == torch.int32 and md.block_pair_offsets.shape == (4, 5)
    finally:
        sys.path.remove(REF)


def test_reference_op_name_is_registered():
    assert hasattr(torch.ops.cuda_sparse_attention, "cuda_bigbird_sparse_attention")
    schema = str(torch.ops.cuda_sparse_attention.cuda_bigbird_sparse_attention.default._schema)
    assert schema.startswith("cuda_sparse_attention::cuda_bigbird_sparse_attention(Tensor q, Tensor k, Tensor v")
