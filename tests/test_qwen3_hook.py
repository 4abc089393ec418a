"""Qwen3 attention hook: config plumbing (CPU) and model-level parity (GPU).

Parity oracle: the same HF Qwen3 model, weights rounded to bf16, run in fp32 on
the CPU with every layer's attention core replaced by the CSR restatement of the
reference's masked attention (oracle.csr_attention over the reference's BigBird
CSR, or full causal attention for dense layers). Tolerance on logits: max-abs
<= 0.1 and >= 95% top-1 agreement (bf16 activations through 2 layers).
"""
from __future__ import annotations

import copy

import numpy as np
import pytest
import torch
from transformers import Qwen3Config
from transformers.models.qwen3.modeling_qwen3 import Qwen3Attention, Qwen3ForCausalLM, apply_rotary_pos_emb

import oracle
from oracle import patterns as op
from sparseattentioninfer_b200 import qwen3 as sq


def tiny_config(**kw):
    cfg = Qwen3Config(vocab_size=512, hidden_size=256, intermediate_size=512, num_hidden_layers=3,
                      num_attention_heads=8, num_key_value_heads=2, head_dim=64, max_position_embeddings=4096,
                      rope_theta=1e6, tie_word_embeddings=False)
    cfg._attn_implementation = "eager"
    for k, v in kw.items():
        setattr(cfg, k, v)
    return cfg


def test_layer_block_experiments_match_reference_logic():
    exps = sq.build_layer_block_experiments(num_layers=36, num_groups=8, layer_span=6, target_sparsity=0.8)
    assert len(exps) == 6
    e = exps[2]
    assert (e["layer_start"], e["layer_end"], e["label"]) == (12, 17, "exp_02_layers_12_17_s0p8")
    assert e["layer_group_sparsities"][12] == [0.8] * 8 and e["layer_group_sparsities"][18] == [0.0] * 8
    assert e["mean_sparsity"] == pytest.approx(0.8 * 6 / 36)


def test_normalization_rejects_bad_values():
    with pytest.raises(ValueError):
        sq.normalize_group_sparsities([0.5, 1.0])
    assert sq.normalize_layer_group_sparsities([None, [0.1]]) == (None, (0.1,))


def _oracle_attention_forward(layouts_by_layer, bs):
    """Forward for Qwen3Attention computing attention with the CPU oracle."""
    def fwd(self, hidden_states, position_embeddings, attention_mask=None, past_key_values=None, **kw):
        shp = hidden_states.shape[:-1]
        hs = (*shp, -1, self.head_dim)
        q = self.q_norm(self.q_proj(hidden_states).view(hs)).transpose(1, 2)
        k = self.k_norm(self.k_proj(hidden_states).view(hs)).transpose(1, 2)
        v = self.v_proj(hidden_states).view(hs).transpose(1, 2)
        cos, sin = position_embeddings
        q, k = apply_rotary_pos_emb(q, k, cos, sin)
        if past_key_values is not None:
            k, v = past_key_values.update(k, v, self.layer_idx)
        H, T_q, T_k = q.shape[1], q.shape[2], k.shape[2]
        lay = layouts_by_layer[self.layer_idx]
        if lay is None:  # dense causal
            lay_eff, bsz = [(bs, 0, -(-T_k // bs), 0)], bs
        else:
            lay_eff, bsz = lay, lay[0][0]
        pairs, offs = op.bigbird_csr(lay_eff, H, T_q, T_k, block_size=bsz)
        out = oracle.csr_attention(q, k, v, pairs, offs, bsz)
        out = out.transpose(1, 2).reshape(*shp, -1)
        return self.o_proj(out), None
    return fwd


@pytest.mark.gpu
def test_sparse_qwen3_matches_oracle_prefill_and_decode(monkeypatch):
    torch.manual_seed(0)
    cfg = tiny_config()
    ref = Qwen3ForCausalLM(cfg).eval()
    for p in ref.parameters():  # the GPU model runs in bf16: give the oracle the same weights
        p.data = p.data.to(torch.bfloat16).float()
    layer_layouts = [[(64, 1, 2, 1), (64, 2, 3, 0)], None, [(64, 1, 1, 2)]]
    sparse = copy.deepcopy(ref).to("cuda", torch.bfloat16)
    sq.replace_qwen3_attention_with_sparse(sparse, layer_layouts=layer_layouts)
    assert all(isinstance(l.self_attn, sq.Qwen3SparseKernelAttention) for l in sparse.model.layers)
    assert sparse.model.layers[1].self_attn.dense
    monkeypatch.setattr(Qwen3Attention, "forward", _oracle_attention_forward(layer_layouts, 64))

    g = torch.Generator().manual_seed(1)
    ids = torch.randint(0, cfg.vocab_size, (2, 300), generator=g)
    with torch.no_grad():
        from transformers import DynamicCache
        cr = DynamicCache()
        lr = ref(ids, past_key_values=cr, use_cache=True).logits
        cs = sq.PreallocatedKVCache(cfg.num_hidden_layers, 512)
        ls = sparse(ids.cuda(), past_key_values=cs, use_cache=True).logits.float().cpu()
        errs = [(ls - lr).abs().max().item()]
        agree = [(ls.argmax(-1) == lr.argmax(-1)).float().mean().item()]
        tok = lr[:, -1].argmax(-1, keepdim=True)
        for _ in range(4):  # greedy decode steps through both caches
            lr1 = ref(tok, past_key_values=cr, use_cache=True).logits
            ls1 = sparse(tok.cuda(), past_key_values=cs, use_cache=True).logits.float().cpu()
            errs.append((ls1 - lr1).abs().max().item())
            agree.append((ls1.argmax(-1) == lr1.argmax(-1)).float().mean().item())
            tok = lr1[:, -1].argmax(-1, keepdim=True)
    assert cs.get_seq_length() == 304
    assert max(errs) <= 0.1, errs
    assert min(agree) >= 0.95, agree
    assert sparse.model.layers[0].self_attn.actual_backend == "cuda_sm100"


@pytest.mark.gpu
@pytest.mark.parametrize("dense_impl", ["sdpa", "cuda_sm100"])
def test_decode_runner_matches_hf_hook(dense_impl):
    """The lean decode runner computes the same decode steps as the HF model with the hook."""
    from sparseattentioninfer_b200.runtime import Qwen3DecodeRunner
    torch.manual_seed(0)
    cfg = tiny_config()
    model = Qwen3ForCausalLM(cfg).to("cuda", torch.bfloat16).eval()
    layer_layouts = [[(64, 1, 2, 1), (64, 2, 3, 0)], None, [(64, 1, 1, 2)]]
    sq.replace_qwen3_attention_with_sparse(model, layer_layouts=layer_layouts)
    ids = torch.randint(0, cfg.vocab_size, (2, 333), generator=torch.Generator().manual_seed(3)).cuda()
    ca, cb = sq.PreallocatedKVCache(3, 400), sq.PreallocatedKVCache(3, 400)
    with torch.no_grad():
        la = model(ids, past_key_values=ca, use_cache=True).logits
        model(ids, past_key_values=cb, use_cache=True)
        runner = Qwen3DecodeRunner(model, cb, layer_layouts, dense_impl=dense_impl)
        tok = la[:, -1].argmax(-1, keepdim=True)
        tb = tok
        for _ in range(4):
            lhf = model(tok, past_key_values=ca, use_cache=True).logits[:, -1].float()
            tb_next, lr = runner.step(tb, return_logits=True)
            assert (lr.float() - lhf).abs().max().item() <= 0.05
            tok = lhf.argmax(-1, keepdim=True)
            tb = tok  # feed both the same token
    assert cb.get_seq_length() == ca.get_seq_length() == 337
