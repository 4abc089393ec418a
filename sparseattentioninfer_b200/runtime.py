"""Lean Qwen3 decode runner over an HF model's weights.

The HF module stack costs ~0.3 ms of host time per layer per decode step
(mask bookkeeping, cache objects, many small ops), which at batch 32 is as much
as the whole GPU step. This runner executes the same decoder arithmetic
(transformers' Qwen3DecoderLayer: RMSNorm, q/k/v projections, per-head q/k
RMSNorm, rotate-half RoPE, attention, o_proj, SwiGLU MLP) with fused
projection weights, a preallocated [B, Hkv, T_max, D] cache written in place,
precomputed RoPE tables and the attention on this package's kernels:

* sparse layers: the split-KV decode kernel over the layer's BigBird CSR, which
  is rebuilt only when T_k crosses a block boundary (the decode row depends on
  (T_k-1)//bs and ceil(T_k/bs) only);
* dense layers: ``dense_impl`` "sdpa" (PyTorch SDPA: library FlashAttention /
  cuDNN, the comparator) or "cuda_sm100" (the decode kernel over a dense CSR).

Prefill goes through the HF model with the hook (``Qwen3SparseKernelAttention``)
and a ``PreallocatedKVCache``; the runner then decodes from that cache.
"""
from __future__ import annotations

import math
from typing import Optional, Sequence

import torch
import torch.nn.functional as F

from . import ops
from .qwen3 import PreallocatedKVCache


class Qwen3DecodeRunner:
    def __init__(self, model, cache: PreallocatedKVCache, layer_layouts: Sequence[Optional[Sequence]],
                 dense_impl: str = "sdpa", n_split: Optional[int] = None):
        cfg = model.config
        self.model = model
        self.cache = cache
        self.H, self.Hkv, self.D = cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim
        self.eps = cfg.rms_norm_eps
        self.layouts = list(layer_layouts)
        self.dense_impl = dense_impl
        self.n_split = n_split
        self.layers = []
        for layer in model.model.layers:
            a, m = layer.self_attn, layer.mlp
            self.layers.append({
                "ln1": layer.input_layernorm.weight, "ln2": layer.post_attention_layernorm.weight,
                "qkv": torch.cat([a.q_proj.weight, a.k_proj.weight, a.v_proj.weight], 0),
                "qn": a.q_norm.weight, "kn": a.k_norm.weight, "o": a.o_proj.weight,
                "gu": torch.cat([m.gate_proj.weight, m.up_proj.weight], 0), "down": m.down_proj.weight,
            })
        self.final_norm = model.model.norm.weight
        self.lm_head = model.lm_head.weight
        self.embed = model.model.embed_tokens.weight
        cap = cache.layers[0].capacity
        dev = self.embed.device
        inv = 1.0 / (cfg.rope_parameters["rope_theta"] if hasattr(cfg, "rope_parameters") and cfg.rope_parameters
                     else cfg.rope_theta) ** (torch.arange(0, self.D, 2, device=dev, dtype=torch.float32) / self.D)
        ang = torch.outer(torch.arange(cap, device=dev, dtype=torch.float32), inv)
        emb = torch.cat([ang, ang], -1)
        self.cos = emb.cos().to(self.embed.dtype)
        self.sin = emb.sin().to(self.embed.dtype)
        self._csr = {}
        self._ws = None

    def _decode_csr(self, li: int, T_k: int):
        lay = self.layouts[li]
        bs = lay[0][0]
        key = (li, (T_k - 1) // bs, math.ceil(T_k / bs))
        hit = self._csr.get(key)
        if hit is None:
            width = max(g + w + r for _, g, w, r in lay)
            hit = ops.compile_bigbird([tuple(x) for x in lay], self.H, 1, T_k, bs, device=self.embed.device,
                                      width=width)
            for k in [k for k in self._csr if k[0] == li]:
                del self._csr[k]
            self._csr[key] = hit
        return hit, bs

    def _dense_csr(self, li: int, T_k: int):
        bs = 128
        nkb = math.ceil(T_k / bs)
        key = (li, "dense", nkb)
        hit = self._csr.get(key)
        if hit is None:
            hit = ops.compile_bigbird([(bs, 0, nkb, 0)], self.H, 1, T_k, bs, device=self.embed.device, width=nkb)
            for k in [k for k in self._csr if k[0] == li]:
                del self._csr[k]
            self._csr[key] = hit
        return hit, bs

    @torch.no_grad()
    def step(self, tok: torch.Tensor, return_logits: bool = False):
        """One greedy decode step for tokens [B, 1]; returns the next tokens [B, 1]
        (and the logits [B, vocab] with ``return_logits``)."""
        B = tok.shape[0]
        H, Hkv, D = self.H, self.Hkv, self.D
        pos = self.cache.layers[0].length
        T_k = pos + 1
        cos, sin = self.cos[pos], self.sin[pos]
        x = F.embedding(tok[:, 0], self.embed)  # [B, hidden]
        if self._ws is None or self._ws[0].numel() < B * H * 64 * D:
            self._ws = (torch.empty(B * H * 64 * D, device=x.device), torch.empty(B * H * 64 * 2, device=x.device))
        for li, L in enumerate(self.layers):
            h = F.rms_norm(x, (x.shape[-1],), L["ln1"], self.eps)
            qkv = h @ L["qkv"].t()
            q = qkv[:, : H * D].view(B, H, D)
            k = qkv[:, H * D: (H + Hkv) * D].view(B, Hkv, D)
            v = qkv[:, (H + Hkv) * D:].view(B, Hkv, D)
            q = F.rms_norm(q, (D,), L["qn"], self.eps)
            k = F.rms_norm(k, (D,), L["kn"], self.eps)
            q = q * cos + torch.cat([-q[..., D // 2:], q[..., : D // 2]], -1) * sin
            k = k * cos + torch.cat([-k[..., D // 2:], k[..., : D // 2]], -1) * sin
            cl = self.cache.layers[li]
            cl.k_buf[:, :, pos].copy_(k)
            cl.v_buf[:, :, pos].copy_(v)
            kv_k, kv_v = cl.k_buf[:, :, :T_k], cl.v_buf[:, :, :T_k]
            q4 = q.unsqueeze(2)  # [B, H, 1, D]
            if self.layouts[li] is not None:
                (pairs, offs), bs = self._decode_csr(li, T_k)
                att = ops.decode_fwd(q4, kv_k, kv_v, pairs, offs, bs, n_split=self.n_split, workspace=self._ws)
            elif self.dense_impl == "sdpa":
                att = F.scaled_dot_product_attention(q4, kv_k, kv_v, enable_gqa=True)
            else:
                (pairs, offs), bs = self._dense_csr(li, T_k)
                att = ops.decode_fwd(q4, kv_k, kv_v, pairs, offs, bs, n_split=self.n_split, workspace=self._ws)
            x = x + att.reshape(B, H * D) @ L["o"].t()
            h = F.rms_norm(x, (x.shape[-1],), L["ln2"], self.eps)
            gu = h @ L["gu"].t()
            inter = gu.shape[-1] // 2
            x = x + (F.silu(gu[:, :inter]) * gu[:, inter:]) @ L["down"].t()
        for cl in self.cache.layers:
            cl.length = T_k
        x = F.rms_norm(x, (x.shape[-1],), self.final_norm, self.eps)
        logits = x @ self.lm_head.t()
        nxt = logits.argmax(-1, keepdim=True)
        return (nxt, logits) if return_logits else nxt
