"""Pin the CPU oracle (oracle/) against fixtures produced by the reference's own code."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from oracle import patterns as op
from tests._inputs import case_inputs, expand_bitmap, layouts_of
from tests.conftest import golden_attn


def _layouts_for(meta):
    kind = meta["kind"]
    T_q, T_k = meta["T_q"], meta["T_k"]
    if kind in ("bigbird_topk", "bigbird2_topk"):
        return [op.bigbird_layout_from_topk(T_k, meta["top_k"])]
    if kind == "keep_ratio":
        return [op.bigbird_layout_from_keep_ratio(T_k, meta["keep_ratio_in"], decode=T_q != T_k)]
    if kind == "group_sparsities":
        decode = T_q != T_k
        krs = [1.0 - s for s in meta["group_sparsities"]]
        shared = op.next_pow2_min16(min(op.bigbird_layout_from_keep_ratio(T_k, kr, decode=decode)[0] for kr in krs))
        return [op.bigbird_layout_from_keep_ratio(T_k, kr, decode=decode, block_size=shared) for kr in krs]
    if kind == "layouts":
        return layouts_of(meta)
    raise KeyError(kind)


BIGBIRD_KINDS = ("bigbird_topk", "bigbird2_topk", "keep_ratio", "group_sparsities", "layouts")


def test_bigbird_csr_matches_reference(manifest, csr_cases):
    n = 0
    for name, meta in manifest["csr"].items():
        if meta["kind"] not in BIGBIRD_KINDS:
            continue
        lay = _layouts_for(meta)
        variant = "bigbird2" if meta["kind"] == "bigbird2_topk" else "bigbird"
        pairs, offs = op.bigbird_csr(lay, meta["H"], meta["T_q"], meta["T_k"], variant=variant)
        np.testing.assert_array_equal(offs, csr_cases[f"{name}.offsets"], err_msg=name)
        np.testing.assert_array_equal(pairs, csr_cases[f"{name}.pairs"], err_msg=name)
        assert meta["block_size"] == op.next_pow2_min16(lay[0][0])
        kr = op.causal_block_keep_ratio(offs, meta["T_q"], meta["T_k"], meta["block_size"])
        assert kr == pytest.approx(meta["keep_ratio"], abs=1e-12), name
        if f"{name}.kvl" in csr_cases:
            kvl = op.bigbird_kv_block_list(lay, meta["H"], meta["T_q"], meta["T_k"], variant=variant)
            np.testing.assert_array_equal(kvl, csr_cases[f"{name}.kvl"], err_msg=name)
        n += 1
    assert n >= 15


def test_token_mask_csr_matches_reference(manifest, csr_cases):
    for name, meta in manifest["csr"].items():
        if meta["kind"] == "token_mask":
            H, T_q, T_k = meta["H"], meta["T_q"], meta["T_k"]
            m = np.unpackbits(csr_cases[f"{name}.mask"], axis=-1)[..., :T_k].astype(bool)
            bm = op.block_bitmap_from_token_mask(torch.from_numpy(m), meta["block_size"])
        elif meta["kind"] == "local":
            m = op.local_window_token_mask(meta["window"], meta["H"], meta["T_q"], meta["T_k"])
            bm = op.block_bitmap_from_token_mask(m, meta["block_size"])
        elif meta["kind"] == "bitmap":
            bm = csr_cases[f"{name}.bitmap"]
        else:
            continue
        pairs, offs = op.csr_from_block_bitmap(bm)
        np.testing.assert_array_equal(offs, csr_cases[f"{name}.offsets"], err_msg=name)
        np.testing.assert_array_equal(pairs, csr_cases[f"{name}.pairs"], err_msg=name)


def test_kv_list_csr_matches_reference(csr_cases):
    pairs, offs = op.csr_from_kv_block_list(csr_cases["kvlist_random.kvl"])
    np.testing.assert_array_equal(offs, csr_cases["kvlist_random.offsets"])
    np.testing.assert_array_equal(pairs, csr_cases["kvlist_random.pairs"])


def _mask_for(meta, csr_cases):
    H, T_q, T_k = meta["H"], meta["T_q"], meta["T_k"]
    if meta["pattern"] == "layouts":
        return op.bigbird_token_mask(layouts_of(meta), H, T_q, T_k)
    if meta["pattern"] == "bitmap":
        bm = csr_cases[f"{meta.get('bitmap', 'cfg1_generator')}.bitmap"]
        return expand_bitmap(bm, meta["block_size"], T_q, T_k)
    raise KeyError(meta["pattern"])


@pytest.mark.parametrize("name", ["cfg1_rotation", "cfg1_generator", "bern_small", "gqa_groups", "decode_gqa",
                                  "ragged_d64"])
def test_masked_sdpa_oracle_matches_reference(name, manifest, csr_cases):
    meta = manifest["attn"][name]
    q, k, v = case_inputs(meta)
    mask = _mask_for(meta, csr_cases)
    rep = meta["H"] // meta["Hkv"]
    out = oracle.masked_sdpa(q, k.repeat_interleave(rep, 1), v.repeat_interleave(rep, 1), mask)
    ref = golden_attn(name)
    np.testing.assert_allclose(out.numpy(), ref, rtol=0, atol=2e-5)
    # chunked restatement (used at full sizes) agrees with the unchunked one
    outc = oracle.masked_sdpa_chunked(q, k, v, lambda h, r0, r1: mask[h, r0:r1], row_chunk=97)
    np.testing.assert_allclose(outc.numpy(), ref, rtol=0, atol=2e-5)


@pytest.mark.parametrize("name", ["cfg1_rotation", "cfg1_generator", "bern_small", "gqa_groups", "decode_gqa",
                                  "ragged_d64"])
def test_csr_attention_matches_masked_reference(name, manifest, csr_cases):
    """The CSR semantics the CUDA kernel implements give the reference's masked-dense output."""
    meta = manifest["attn"][name]
    q, k, v = case_inputs(meta)
    bs = meta["block_size"]
    if meta["pattern"] == "layouts":
        pairs, offs = op.bigbird_csr(layouts_of(meta), meta["H"], meta["T_q"], meta["T_k"])
    else:
        bm = csr_cases[f"{meta.get('bitmap', 'cfg1_generator')}.bitmap"]
        pairs, offs = op.csr_from_block_bitmap(bm)
    out = oracle.csr_attention(q, k, v, pairs, offs, bs, row_chunk=256)
    np.testing.assert_allclose(out.numpy(), golden_attn(name), rtol=0, atol=2e-5)
