"""Qwen3 through the reference's masked-dense attention path — TEST INFRASTRUCTURE ONLY.

Restates, in fp32 on the host, what the reference's sparse Qwen3 computes for a
prompt: transformers' Qwen3 decoder arithmetic (RMSNorm, q/k/v projections,
per-head q/k RMSNorm, rotate-half RoPE, repeat_kv, o_proj, SwiGLU MLP;
sparse_llm/qwen3/integrations/modeling_sparse_qwen3.py:200-260) with attention
from MaskedSdpaBackend over the BigBird token mask
(sparse_attentions/attention/masked_sdpa.py:23-68,
sparse_attentions/patterns/bigbird_pattern.py:487-531).

``CheckerKernels`` offers the pattern, attention and layer-step calls of the CUDA
ops module (compile_bigbird, prefill_fwd, decode_fwd, qk_norm_rope_append,
add_rms_norm, silu_mul) computed by this oracle, so that the tensor-parallel host
logic can be exercised on CPU ranks (gloo) without a GPU.
"""
from __future__ import annotations

import math

import numpy as np
import torch
import torch.nn.functional as F

from .attention import csr_attention, masked_sdpa
from .patterns import bigbird_csr, bigbird_token_mask


def _rms(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    # Qwen3RMSNorm: normalise in fp32, back to the activation dtype, times the weight
    xf = x.float()
    return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)).to(x.dtype) * w


def _rope(x: torch.Tensor, theta: float, offset: int = 0) -> torch.Tensor:
    # apply_rotary_pos_emb: fp32 angles, cos/sin in the activation dtype
    T, D = x.shape[-2], x.shape[-1]
    inv = 1.0 / theta ** (torch.arange(0, D, 2, dtype=torch.float32, device=x.device) / D)
    ang = torch.outer(torch.arange(offset, offset + T, dtype=torch.float32, device=x.device), inv)
    emb = torch.cat([ang, ang], -1)
    rot = torch.cat([-x[..., D // 2:], x[..., : D // 2]], -1)
    return x * emb.cos().to(x.dtype) + rot * emb.sin().to(x.dtype)


@torch.no_grad()
def masked_dense_forward(weights, tokens: torch.Tensor, layout, sparse_layers=None, cache=None,
                         device="cpu", dtype=torch.float32) -> torch.Tensor:
    """Logits of the last position [B, vocab] (fp32) for ``tokens`` [B, T_new]
    appended to ``cache`` (a list of per-layer (k, v) fp32 tensors [B, Hkv, T, D],
    extended in place; None = empty prompt). Weights are a one-rank set (fields as
    in sparseattentioninfer_b200.tp.Qwen3TPWeights, world 1). Sparse layers use the
    BigBird token mask of (T_new, T_total) as the hook builds it; the others dense
    causal attention. ``device`` only says where the torch arithmetic runs (a
    full-width model checks faster on a GPU); the computation is the same.
    ``dtype`` bfloat16 runs the same model with bf16 weights and activations (the
    reference model as deployed; attention scores and softmax stay fp32, as in
    masked_sdpa), to size the rounding error of bf16 itself."""
    A = weights.arch
    f = lambda t: t.detach().to(device=device, dtype=dtype)  # noqa: E731
    B, T = tokens.shape
    H, Hkv, D = A.heads, A.kv_heads, A.head_dim
    rep = H // Hkv
    past = 0 if not cache else cache[0][0].shape[2]
    x = f(weights.embed)[tokens.to(device)]
    mask = torch.as_tensor(bigbird_token_mask([tuple(layout)], H, T, past + T)).to(device)
    sparse = set(range(A.layers)) if sparse_layers is None else set(sparse_layers)
    for li, L in enumerate(weights.layers):
        h = _rms(x, f(L["ln1"]), A.eps)
        qkv = h @ f(L["qkv"]).t()
        q = qkv[..., : H * D].view(B, T, H, D).transpose(1, 2)
        k = qkv[..., H * D:(H + Hkv) * D].view(B, T, Hkv, D).transpose(1, 2)
        v = qkv[..., (H + Hkv) * D:].view(B, T, Hkv, D).transpose(1, 2)
        q = _rope(_rms(q, f(L["qn"]), A.eps), A.rope_theta, past)
        k = _rope(_rms(k, f(L["kn"]), A.eps), A.rope_theta, past)
        if cache is not None:
            if len(cache) <= li:
                cache.append((k, v))
            else:
                k = torch.cat([cache[li][0], k], 2)
                v = torch.cat([cache[li][1], v], 2)
                cache[li] = (k, v)
        kr, vr = k.repeat_interleave(rep, 1), v.repeat_interleave(rep, 1)
        if li in sparse:
            att = masked_sdpa(q, kr, vr, mask, "mask").to(dtype)
        elif T == 1:
            att = masked_sdpa(q, kr, vr, torch.ones(H, 1, kr.shape[2], dtype=torch.bool, device=device), "mask")
        else:
            att = masked_sdpa(q, kr, vr, torch.ones(H, T, kr.shape[2], dtype=torch.bool, device=device), "mask")
        att = att.to(dtype)
        x = x + att.transpose(1, 2).reshape(B, T, H * D) @ f(L["o"]).t()
        h = _rms(x, f(L["ln2"]), A.eps)
        gu = h @ f(L["gu"]).t()
        inter = gu.shape[-1] // 2
        x = x + (F.silu(gu[..., :inter]) * gu[..., inter:]) @ f(L["down"]).t()
    x = _rms(x[:, -1], f(weights.final_norm), A.eps)
    return (x @ f(weights.lm_head).t()).float().cpu()


def masked_dense_last_logits(weights, tokens: torch.Tensor, layout, sparse_layers=None) -> torch.Tensor:
    """``masked_dense_forward`` of a whole prompt without a cache."""
    return masked_dense_forward(weights, tokens, layout, sparse_layers)


class CheckerKernels:
    """The CUDA ops' pattern/attention calls restated on the host (fp32)."""

    @staticmethod
    def compile_bigbird(layouts, n_heads, T_q, T_k, block_size, *, variant=None, device="cpu", width=None):
        pairs, offs = bigbird_csr([tuple(l) for l in layouts], n_heads, T_q, T_k, block_size=block_size)
        if width is not None:
            if pairs.shape[1] > width and int(np.diff(offs, axis=1).sum(1).max()) > width:
                raise ValueError("width below the row length")
            p = np.zeros((n_heads, width), dtype=np.int32)
            n = min(width, pairs.shape[1])
            p[:, :n] = pairs[:, :n]
            pairs = p
        return torch.from_numpy(pairs).to(device), torch.from_numpy(offs).to(device)

    @staticmethod
    def prefill_fwd(q, k, v, block_pairs, block_pair_offsets, block_size, *, scale=None, out=None):
        o = csr_attention(q.float().cpu(), k.float().cpu(), v.float().cpu(), block_pairs.cpu().numpy(),
                          block_pair_offsets.cpu().numpy(), block_size)
        if out is None:
            return o.to(q.dtype)
        out.copy_(o)
        return out

    @staticmethod
    def qk_norm_rope_append(qkv, q_weight, k_weight, cos, sin, k_cache, v_cache, *, Hq, Hkv, pos=0, pos_dev=None,
                            eps=1e-6, q_out=None):
        p = int(pos_dev.item()) if pos_dev is not None else int(pos)
        B, T, _, D = qkv.shape
        x = qkv.float()
        c = cos[p:p + T].float().view(1, T, 1, D)
        s = sin[p:p + T].float().view(1, T, 1, D)

        def norm_rope(t, w):
            t = _rms(t, w.float(), eps)
            return t * c + torch.cat([-t[..., D // 2:], t[..., : D // 2]], -1) * s

        q = norm_rope(x[:, :, :Hq], q_weight)
        k = norm_rope(x[:, :, Hq:Hq + Hkv], k_weight)
        k_cache[:, :, p:p + T] = k.transpose(1, 2).to(k_cache.dtype)
        v_cache[:, :, p:p + T] = x[:, :, Hq + Hkv:].transpose(1, 2).to(v_cache.dtype)
        return q.to(qkv.dtype).transpose(1, 2)

    @staticmethod
    def add_rms_norm(x, y, weight, eps=1e-6, out=None):
        if y is not None:
            x += y
        o = _rms(x.float(), weight.float(), eps).to(x.dtype)
        if out is None:
            return o
        out.copy_(o)
        return out

    @staticmethod
    def silu_mul(gate_up, out=None):
        inter = gate_up.shape[-1] // 2
        g = gate_up.float()
        o = (F.silu(g[..., :inter]) * g[..., inter:]).to(gate_up.dtype)
        if out is None:
            return o
        out.copy_(o)
        return out

    @staticmethod
    def linear_m8(x, weight, out=None, *, glu=False):
        if glu:
            n = weight.shape[0] // 2
            g = (x.float() @ weight[:n].float().t()).to(x.dtype).float()
            u = (x.float() @ weight[n:].float().t()).to(x.dtype).float()
            o = (F.silu(g) * u).to(x.dtype)
        else:
            o = (x.float() @ weight.float().t()).to(x.dtype)
        if out is None:
            return o
        out.copy_(o)
        return out

    @staticmethod
    def decode_fwd(q, k, v, block_pairs, block_pair_offsets, block_size, *, scale=None, n_split=None, out=None,
                   workspace=None):
        return CheckerKernels.prefill_fwd(q, k, v, block_pairs, block_pair_offsets, block_size, out=out)


__all__ = ["masked_dense_forward", "masked_dense_last_logits", "CheckerKernels"]
