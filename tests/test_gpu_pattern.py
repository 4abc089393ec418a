"""Device pattern compiler vs the reference's CSR (golden fixtures), bit-exact."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import sparseattentioninfer_b200 as sa
from sparseattentioninfer_b200 import _capi, ops
from tests._inputs import layouts_of

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _pattern_for(meta):
    kind, H = meta["kind"], meta.get("H")
    kw = dict(exact_width=True, build_kv_block_list=True)
    if kind == "bigbird_topk":
        return sa.BigBirdPattern(top_k=meta["top_k"], n_heads=H, **kw)
    if kind == "bigbird2_topk":
        return sa.BigBird2Pattern(top_k=meta["top_k"], n_heads=H, **kw)
    if kind == "keep_ratio":
        return sa.BigBirdKeepRatioPattern(keep_ratio=meta["keep_ratio_in"], n_heads=H, **kw)
    if kind == "group_sparsities":
        return sa.BigBirdKeepRatioPattern(group_sparsities=meta["group_sparsities"], n_heads=H,
                                          n_kv_heads=meta["n_kv_heads"], **kw)
    if kind == "layouts":
        return sa.BigBirdKeepRatioPattern(layouts=layouts_of(meta), n_heads=H, **kw)
    return None


def test_bigbird_family_bit_exact(manifest, csr_cases):
    n = 0
    for name, meta in manifest["csr"].items():
        pat = _pattern_for(meta)
        if pat is None:
            continue
        q = torch.empty(1, meta["H"], meta["T_q"], 8, device=DEV)
        k = torch.empty(1, meta["H"], meta["T_k"], 8, device=DEV)
        md = pat.build(q, k)
        np.testing.assert_array_equal(md.block_pair_offsets.cpu().numpy(), csr_cases[f"{name}.offsets"], err_msg=name)
        np.testing.assert_array_equal(md.block_pairs.cpu().numpy(), csr_cases[f"{name}.pairs"], err_msg=name)
        assert md.block_size == meta["block_size"]
        assert md.keep_ratio == pytest.approx(meta["keep_ratio"], abs=1e-12)
        if f"{name}.kvl" in csr_cases:
            np.testing.assert_array_equal(md.kv_block_list.cpu().numpy(), csr_cases[f"{name}.kvl"], err_msg=name)
        n += 1
    assert n >= 15
    assert _capi.device_error() == 0


def test_decode_no_sync_width_is_a_bound(manifest, csr_cases):
    meta = manifest["csr"]["cfg4_decode"]
    pat = sa.BigBirdKeepRatioPattern(layouts=layouts_of(meta), n_heads=meta["H"])  # decode: sync-free width
    md = pat.build(torch.empty(1, 32, 1, 8, device=DEV), torch.empty(1, 32, meta["T_k"], 8, device=DEV))
    offs = md.block_pair_offsets.cpu().numpy()
    np.testing.assert_array_equal(offs, csr_cases["cfg4_decode.offsets"])
    ref = csr_cases["cfg4_decode.pairs"]
    got = md.block_pairs.cpu().numpy()
    assert got.shape[1] >= ref.shape[1]
    for h in range(32):
        np.testing.assert_array_equal(got[h, : offs[h, -1]], ref[h, : offs[h, -1]])


def test_token_mask_and_bitmap_bit_exact(manifest, csr_cases):
    for name, meta in manifest["csr"].items():
        if meta["kind"] == "token_mask":
            T_k = meta["T_k"]
            m = np.unpackbits(csr_cases[f"{name}.mask"], axis=-1)[..., :T_k].astype(bool)
            pairs, offs = ops.compile_token_mask(torch.from_numpy(m).to(DEV), meta["block_size"])
        elif meta["kind"] == "local":
            pat = sa.LocalWindowPattern(window_size=meta["window"], block_size=meta["block_size"])
            md = pat.build(torch.empty(1, 2, meta["T_q"], 8, device=DEV), torch.empty(1, 2, meta["T_k"], 8, device=DEV))
            pairs, offs = md.block_pairs, md.block_pair_offsets
        elif meta["kind"] == "bitmap":
            pairs, offs = ops.compile_block_bitmap(torch.from_numpy(csr_cases[f"{name}.bitmap"]).to(DEV))
        else:
            continue
        np.testing.assert_array_equal(offs.cpu().numpy(), csr_cases[f"{name}.offsets"], err_msg=name)
        np.testing.assert_array_equal(pairs.cpu().numpy(), csr_cases[f"{name}.pairs"], err_msg=name)


def test_kv_block_list_bit_exact(csr_cases):
    pairs, offs = ops.compile_kv_block_list(torch.from_numpy(csr_cases["kvlist_random.kvl"]).to(DEV))
    np.testing.assert_array_equal(offs.cpu().numpy(), csr_cases["kvlist_random.offsets"])
    np.testing.assert_array_equal(pairs.cpu().numpy(), csr_cases["kvlist_random.pairs"])


def test_full_size_bigbird_against_oracle():
    """BASELINE-size layouts: device CSR == host restatement (pinned above)."""
    from oracle import patterns as op
    from sparseattentioninfer_b200 import workloads as wl
    for layouts, H, T in [(wl.config3_group_layouts(), 32, 16384), ([(128, 2, 4, 3)], 32, 65536),
                          ([(64, 2, 4, 2)], 32, 32768)]:
        pairs, offs = ops.compile_bigbird(layouts, H, T, T, layouts[0][0], device=DEV)
        rp, ro = op.bigbird_csr(layouts, H, T, T)
        np.testing.assert_array_equal(offs.cpu().numpy(), ro)
        np.testing.assert_array_equal(pairs.cpu().numpy(), rp)


@pytest.mark.gpu
@pytest.mark.parametrize("layouts,H,bs", [([(64, 2, 4, 2)], 32, 64), ([(128, 2, 4, 3)], 32, 128),
                                          ([(64, 1, 2, 3), (64, 3, 5, 1)], 8, 64), ([(64, 0, 1 << 30, 0)], 4, 64)])
def test_device_decode_rows_match_host_compiled_rows(layouts, H, bs):
    """sa_bigbird_decode_row with the key count on the device gives the decode rows
    compile_bigbird builds for T_q = 1, for lengths across block boundaries and
    for a head sub-range (a tensor-parallel rank's rows)."""
    from sparseattentioninfer_b200 import ops
    width = 4096 // bs + 8 if layouts[0][2] >= (1 << 29) else max(g + w + r for _, g, w, r in layouts)
    lo, n = (H // 2, H // 2)
    for T_k in [1, bs - 1, bs, bs + 1, 3 * bs, 3 * bs + 7, 4000]:
        sl = torch.tensor([T_k], dtype=torch.int32, device="cuda:0")
        gp = torch.full((n, width), -7, dtype=torch.int32, device="cuda:0")
        go = torch.zeros(n, 2, dtype=torch.int32, device="cuda:0")
        ops.bigbird_decode_row(layouts, H, sl, bs, gp, go, head_lo=lo)
        hp, ho = ops.compile_bigbird(layouts, H, 1, T_k, bs, device="cuda:0")
        for i in range(n):
            a, b = int(go[i, 1]), int(ho[lo + i, 1] - ho[lo + i, 0])
            assert int(go[i, 0]) == 0 and a == b, (T_k, i)
            assert torch.equal(gp[i, :a], hp[lo + i, int(ho[lo + i, 0]):int(ho[lo + i, 1])]), (T_k, i)
