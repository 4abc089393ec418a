"""Qwen3 attention hook: HF ``Qwen3Attention`` with the attention core on the B200 kernels.

Mirrors sparse_llm/qwen3/integrations/modeling_sparse_qwen3.py
(``Qwen3SparseKernelAttention`` :93-315, ``replace_qwen3_attention_with_sparse``
:347-406, ``Qwen3SparseKernelForCausalLM`` :470-484) and the layer-block
selection of sparse_llm/qwen3/experiment/layer_block_sparsity.py:193-223, with
these deliberate differences:

* ``forward`` takes transformers-5.x ``past_key_values`` (the reference's
  ``past_key_value`` argument never receives the cache under transformers 5.x,
  so its decode ran without one);
* K/V keep their Hkv heads (no ``repeat_kv`` copy): the kernels read KV head
  h // (Hq/Hkv);
* a layer without a sparsity entry is truly dense (full causal attention via a
  dense block CSR), whereas the reference's "0.0 sparsity" is still BigBird;
* explicit per-group BigBird layouts per layer (``sparse_attention_layer_layouts``)
  are accepted, the supported form of the reference's ``_layout_cache``
  injection;
* no fallback: the attention runs on the CUDA backend or raises.

``PreallocatedKVCache`` is a transformers ``Cache`` whose layers hold a
fixed-capacity [B, Hkv, T_max, D] buffer and return [:, :, :T] views, replacing
the ``torch.cat`` growth of DynamicCache (one O(T) copy per step per layer).
"""
from __future__ import annotations

from typing import Any, Optional, Sequence

import torch
from torch import nn
from transformers.cache_utils import Cache, DynamicLayer
from transformers.models.qwen3.configuration_qwen3 import Qwen3Config
from transformers.models.qwen3.modeling_qwen3 import Qwen3Attention, Qwen3ForCausalLM, apply_rotary_pos_emb

from . import ops as _ops
from .backend import CudaSm100Backend
from .patterns import (
    BigBirdKeepRatioPattern,
    BigBirdPattern,
    DenseCausalPattern,
    LocalWindowPattern,
    SparsePattern,
)


ATTN_IMPLEMENTATION = "cuda_sm100"


def _no_mask(*args, **kwargs):
    """The kernels apply causality (and padding is unsupported, as in the
    reference hook): no [B, 1, T_q, T_k] mask is materialised."""
    return None


def _attention_interface(module, query, key, value, attention_mask, **kwargs):
    raise RuntimeError("layers using the cuda_sm100 implementation must be Qwen3SparseKernelAttention")


def register_attention_implementation() -> str:
    """Register ``cuda_sm100`` with transformers' attention and mask interfaces so a
    model config can name it (``config._attn_implementation = "cuda_sm100"``):
    mask creation is then skipped entirely."""
    from transformers.masking_utils import ALL_MASK_ATTENTION_FUNCTIONS
    from transformers.modeling_utils import ALL_ATTENTION_FUNCTIONS
    ALL_MASK_ATTENTION_FUNCTIONS.register(ATTN_IMPLEMENTATION, _no_mask)
    ALL_ATTENTION_FUNCTIONS.register(ATTN_IMPLEMENTATION, _attention_interface)
    return ATTN_IMPLEMENTATION


def _get(config, name: str, default):
    return getattr(config, name, default)


def normalize_group_sparsities(values, *, name: str = "group_sparsities"):
    """sparse_config.py:20-27."""
    if values is None:
        return None
    out = tuple(float(v) for v in values)
    if any(not 0.0 <= v < 1.0 for v in out):
        raise ValueError(f"{name} values must satisfy 0 <= sparsity < 1.")
    return out


def normalize_layer_group_sparsities(values, *, name: str = "layer_group_sparsities"):
    """sparse_config.py:30-48."""
    if values is None:
        return None
    return tuple(None if v is None else normalize_group_sparsities(v, name=f"{name}[{i}]")
                 for i, v in enumerate(values))


def build_layer_block_experiments(*, num_layers: int, num_groups: int, layer_span: int,
                                  target_sparsity: float) -> list[dict[str, Any]]:
    """layer_block_sparsity.py:193-223: contiguous blocks of ``layer_span`` layers get
    ``target_sparsity`` in every KV group, the other layers 0.0."""
    exps = []
    for idx, start in enumerate(range(0, num_layers, layer_span)):
        stop = min(start + layer_span, num_layers)
        lgs = [[target_sparsity if start <= li < stop else 0.0] * num_groups for li in range(num_layers)]
        mean = sum(v for row in lgs for v in row) / max(1, num_layers * num_groups)
        slug = f"{target_sparsity:g}".replace(".", "p")
        exps.append({"experiment_idx": idx, "label": f"exp_{idx:02d}_layers_{start}_{stop - 1}_s{slug}",
                     "layer_start": start, "layer_end": stop - 1, "layer_count": stop - start,
                     "target_sparsity": target_sparsity, "mean_sparsity": mean,
                     "layer_group_sparsities": lgs})
    return exps


class Qwen3SparseKernelAttention(Qwen3Attention):
    """HF Qwen3 attention with the attention core replaced by the cuda_sm100 backend."""

    def __init__(self, config: Qwen3Config, layer_idx: int, *, backend_name: Optional[str] = None,
                 window_size: Optional[int] = None, block_size: Optional[int] = None, group_sparsities=None,
                 layouts: Optional[Sequence[Sequence[int]]] = None, dense: Optional[bool] = None):
        super().__init__(config, layer_idx)
        self.num_heads = config.num_attention_heads
        self.num_key_value_heads = config.num_key_value_heads
        self.pattern_name = _get(config, "sparse_attention_pattern", "local")
        requested = backend_name or _get(config, "sparse_attention_backend", "auto")
        if requested not in ("auto", "cuda_sm100"):
            raise ValueError(f"backend {requested!r} unavailable: this package provides 'cuda_sm100' only")
        self.backend_name = "cuda_sm100"
        self.window_size = window_size or _get(config, "sparse_attention_window_size", 512)
        self.block_size = block_size or _get(config, "sparse_attention_block_size", 64)
        self.top_k = _get(config, "sparse_attention_top_k", 128)
        keep_ratio = _get(config, "sparse_attention_keep_ratio", None)
        gs = normalize_group_sparsities(group_sparsities)
        if layouts is None:
            lay_cfg = _get(config, "sparse_attention_layer_layouts", None)
            if lay_cfg is not None and layer_idx < len(lay_cfg):
                layouts = lay_cfg[layer_idx]
                if layouts is None and dense is None:
                    dense = True
        if gs is None and layouts is None:
            lgs = normalize_layer_group_sparsities(_get(config, "sparse_attention_layer_group_sparsities", None))
            if lgs is not None and layer_idx < len(lgs):
                gs = lgs[layer_idx]
        if gs is None and layouts is None:
            gs = normalize_group_sparsities(_get(config, "sparse_attention_group_sparsities", None))
        self.group_sparsities = gs
        self.keep_ratio = None if gs is not None else keep_ratio
        self.dense = bool(dense) or self.pattern_name == "dense"
        self.sparse_backend = CudaSm100Backend()
        self.sparse_pattern = self._make_pattern(layouts)
        self.last_pattern_stats: Optional[dict] = None
        self.collect_pattern_stats = True
        # Dense layers run the cuda_sm100 kernel over a dense causal CSR; "sdpa"
        # selects PyTorch SDPA (library FlashAttention / cuDNN), the comparator
        # the reference's benchmarks call the dense path.
        self.dense_impl = _get(config, "sparse_attention_dense_impl", "cuda_sm100")
        # The fused prologue (one projection GEMM + ops.qk_norm_rope_append) serves
        # a PreallocatedKVCache when RoPE is the default kind and there is no bias.
        rope = _get(config, "rope_parameters", None) or {}
        self._rope_theta = float(rope.get("rope_theta", _get(config, "rope_theta", 10000.0)))
        self._fusable = (rope.get("rope_type", "default") == "default" and self.q_proj.bias is None
                         and self.head_dim in (64, 128))
        self._qkv_cache = None
        self._rope_tab = None

    @property
    def actual_backend(self) -> str:
        return self.sparse_backend.actual_backend

    def set_dense(self, dense: bool = True, impl: Optional[str] = None) -> None:
        """Switch this layer to full causal attention (or back to its pattern)."""
        if impl is not None:
            self.dense_impl = impl
        if dense:
            self.dense = True
            self.sparse_pattern = DenseCausalPattern()

    def _make_pattern(self, layouts) -> SparsePattern:
        H, Hkv = self.num_heads, self.num_key_value_heads
        if self.dense:
            return DenseCausalPattern()
        if layouts is not None:
            return BigBirdKeepRatioPattern(layouts=[tuple(l) for l in layouts], n_heads=H)
        if self.pattern_name == "bigbird":
            if self.group_sparsities is not None:
                return BigBirdKeepRatioPattern(group_sparsities=self.group_sparsities, n_heads=H, n_kv_heads=Hkv)
            if self.keep_ratio is not None:
                return BigBirdKeepRatioPattern(keep_ratio=self.keep_ratio, n_heads=H, n_kv_heads=Hkv)
            return BigBirdPattern(top_k=self.top_k, n_heads=H)
        return LocalWindowPattern(window_size=self.window_size, block_size=self.block_size, materialize_mask=False)

    def _fused_qkv_weight(self) -> torch.Tensor:
        """[Wq; Wk; Wv] as one matrix: a view when the three weights are adjacent
        slices of one buffer (e.g. hf_model_over_tp), else a copy made once."""
        wq, wk, wv = self.q_proj.weight, self.k_proj.weight, self.v_proj.weight
        key = (wq.data_ptr(), wk.data_ptr(), wv.data_ptr(), wq._version, wk._version, wv._version)
        if self._qkv_cache is not None and self._qkv_cache[0] == key:
            return self._qkv_cache[1]
        es = wq.element_size()
        adjacent = (wq.is_contiguous() and wk.is_contiguous() and wv.is_contiguous()
                    and wq.untyped_storage().data_ptr() == wk.untyped_storage().data_ptr()
                    == wv.untyped_storage().data_ptr()
                    and wk.data_ptr() == wq.data_ptr() + wq.numel() * es
                    and wv.data_ptr() == wk.data_ptr() + wk.numel() * es)
        if adjacent:
            fused = torch.empty(0, dtype=wq.dtype, device=wq.device).set_(
                wq.untyped_storage(), wq.storage_offset(), (wq.shape[0] + wk.shape[0] + wv.shape[0], wq.shape[1]),
                (wq.shape[1], 1))
        else:
            fused = torch.cat([wq, wk, wv], 0)
        self._qkv_cache = (key, fused)
        return fused

    def _rope_tables(self, capacity: int, device, dtype):
        """cos / sin [capacity, D] of the default RoPE (fp32 angles, stored in the
        activation dtype), as apply_rotary_pos_emb uses them."""
        t = self._rope_tab
        if t is None or t[0].shape[0] < capacity or t[0].device != device or t[0].dtype != dtype:
            D = self.head_dim
            inv = 1.0 / self._rope_theta ** (torch.arange(0, D, 2, device=device, dtype=torch.float32) / D)
            ang = torch.outer(torch.arange(capacity, device=device, dtype=torch.float32), inv)
            emb = torch.cat([ang, ang], -1)
            t = self._rope_tab = (emb.cos().to(dtype), emb.sin().to(dtype))
        return t

    def _fused_prologue(self, hidden_states: torch.Tensor, cache: "PreallocatedKVCache"):
        """q/k RMSNorm + RoPE + the append of k/v to the preallocated cache in one
        kernel (ops.qk_norm_rope_append) after one fused projection GEMM, in place
        of q_norm / k_norm / apply_rotary_pos_emb / cache.update
        (modeling_sparse_qwen3.py:211-231). Returns q [B, Hq, T, D] and the cache's
        k / v views [B, Hkv, length, D]."""
        B, T, _ = hidden_states.shape
        H, Hkv, D = self.num_heads, self.num_key_value_heads, self.head_dim
        cl = cache.layers[self.layer_idx]
        if not cl.is_initialized:
            z = torch.empty(B, Hkv, 0, D, dtype=hidden_states.dtype, device=hidden_states.device)
            cl.lazy_initialization(z, z)
        if cl.length + T > cl.capacity:
            raise RuntimeError(f"KV cache capacity {cl.capacity} exceeded")
        qkv = (hidden_states @ self._fused_qkv_weight().t()).view(B, T, H + 2 * Hkv, D)
        cos, sin = self._rope_tables(cl.capacity, qkv.device, qkv.dtype)
        q = _ops.qk_norm_rope_append(qkv, self.q_norm.weight, self.k_norm.weight, cos, sin, cl.k_buf, cl.v_buf,
                                     Hq=H, Hkv=Hkv, pos=cl.length, eps=self.q_norm.variance_epsilon)
        cl.length += T
        cl.keys, cl.values = cl.k_buf[:, :, :cl.length], cl.v_buf[:, :, :cl.length]
        return q, cl.keys, cl.values

    def forward(self, hidden_states: torch.Tensor, position_embeddings: tuple[torch.Tensor, torch.Tensor],
                attention_mask: Optional[torch.Tensor] = None, past_key_values: Optional[Cache] = None, **kwargs):
        if kwargs.get("output_attentions", False):
            raise NotImplementedError("Sparse kernel path does not return attention weights.")
        input_shape = hidden_states.shape[:-1]
        hidden_shape = (*input_shape, -1, self.head_dim)
        if self._fusable and isinstance(past_key_values, PreallocatedKVCache) and \
                hidden_states.dtype == torch.bfloat16 and hidden_states.is_cuda:
            q, k, v = self._fused_prologue(hidden_states, past_key_values)
        else:
            q = self.q_norm(self.q_proj(hidden_states).view(hidden_shape)).transpose(1, 2)
            k = self.k_norm(self.k_proj(hidden_states).view(hidden_shape)).transpose(1, 2)
            v = self.v_proj(hidden_states).view(hidden_shape).transpose(1, 2)
            cos, sin = position_embeddings
            q, k = apply_rotary_pos_emb(q, k, cos, sin)
            if past_key_values is not None:
                k, v = past_key_values.update(k, v, self.layer_idx)
        if self.dense and self.dense_impl == "sdpa" and q.shape[2] in (1, k.shape[2]):
            # (SDPA aligns its causal mask top-left, so chunked prefill, 1 < T_q < T_k,
            # stays on the cuda_sm100 kernel, whose mask is bottom-right aligned.)
            T_q = q.shape[2]
            out = torch.nn.functional.scaled_dot_product_attention(q, k, v, is_causal=T_q > 1, enable_gqa=True)
            out = out.transpose(1, 2).reshape(*input_shape, -1).contiguous()
            return self.o_proj(out), None
        pattern = self.sparse_pattern.build(q, k, causal=True)
        if self.collect_pattern_stats:
            kr = pattern.keep_ratio
            self.last_pattern_stats = {"keep_ratio": float(kr), "sparsity": 1.0 - float(kr)}
        out = self.sparse_backend.forward(q, k, v, pattern)
        out = out.transpose(1, 2).reshape(*input_shape, -1).contiguous()
        return self.o_proj(out), None


def build_sparse_attention_from_dense(attention: nn.Module, **kw) -> Qwen3SparseKernelAttention:
    """modeling_sparse_qwen3.py:320-344: same weights, sparse core."""
    target_dtype = kw.pop("target_dtype", None)
    sa = Qwen3SparseKernelAttention(attention.config, layer_idx=attention.layer_idx, **kw)
    sa.load_state_dict(attention.state_dict(), strict=False)
    sa.to(device=attention.q_proj.weight.device, dtype=target_dtype or attention.q_proj.weight.dtype)
    return sa


def replace_qwen3_attention_with_sparse(model: nn.Module, *, block_size: int = 64, group_sparsities=None,
                                        layer_group_sparsities=None, layer_layouts=None,
                                        target_dtype=None, **kw) -> nn.Module:
    """modeling_sparse_qwen3.py:347-406. ``layer_layouts[i]`` (a list of per-group
    (bs, g, w, r) layouts, or None for a dense layer) overrides the sparsities."""
    base = model.model if hasattr(model, "model") and hasattr(model.model, "layers") else model
    if not hasattr(base, "layers"):
        raise TypeError("Expected a Qwen3 decoder model with a `.layers` attribute.")
    gs = normalize_group_sparsities(group_sparsities)
    lgs = normalize_layer_group_sparsities(layer_group_sparsities)
    if lgs is not None and len(lgs) > len(base.layers):
        raise ValueError("layer_group_sparsities has more entries than there are decoder layers.")
    if layer_layouts is not None and len(layer_layouts) > len(base.layers):
        raise ValueError("layer_layouts has more entries than there are decoder layers.")
    for layer in base.layers:
        li = layer.self_attn.layer_idx
        args = dict(kw, block_size=block_size, target_dtype=target_dtype)
        if layer_layouts is not None and li < len(layer_layouts):
            if layer_layouts[li] is None:
                args["dense"] = True
            else:
                args["layouts"] = layer_layouts[li]
        else:
            layer_gs = lgs[li] if lgs is not None and li < len(lgs) else None
            args["group_sparsities"] = layer_gs if layer_gs is not None else gs
        layer.self_attn = build_sparse_attention_from_dense(layer.self_attn, **args)
    return model


class Qwen3SparseKernelForCausalLM(Qwen3ForCausalLM):
    """modeling_sparse_qwen3.py:470-484: every layer's attention is replaced at construction."""

    def __init__(self, config: Qwen3Config, *, group_sparsities=None, layer_group_sparsities=None,
                 layer_layouts=None):
        if not hasattr(config, "_attn_implementation") or config._attn_implementation is None:
            config._attn_implementation = "eager"
        super().__init__(config)
        replace_qwen3_attention_with_sparse(
            self.model, block_size=_get(config, "sparse_attention_block_size", 64),
            group_sparsities=group_sparsities if group_sparsities is not None
            else _get(config, "sparse_attention_group_sparsities", None),
            layer_group_sparsities=layer_group_sparsities if layer_group_sparsities is not None
            else _get(config, "sparse_attention_layer_group_sparsities", None),
            layer_layouts=layer_layouts if layer_layouts is not None
            else _get(config, "sparse_attention_layer_layouts", None))


class PreallocatedLayer(DynamicLayer):
    """KV layer with a fixed [B, Hkv, capacity, D] buffer; ``update`` writes the new
    tokens in place and returns [:, :, :T] views (no per-step concatenation)."""

    def __init__(self, capacity: int):
        super().__init__()
        self.capacity = capacity
        self.length = 0

    def lazy_initialization(self, key_states, value_states):
        self.dtype, self.device = key_states.dtype, key_states.device
        B, H, _, D = key_states.shape
        self.k_buf = torch.empty(B, H, self.capacity, D, dtype=self.dtype, device=self.device)
        self.v_buf = torch.empty(B, H, self.capacity, D, dtype=self.dtype, device=self.device)
        self.keys, self.values = self.k_buf[:, :, :0], self.v_buf[:, :, :0]
        self.is_initialized = True

    def update(self, key_states, value_states, *args, **kwargs):
        if not self.is_initialized:
            self.lazy_initialization(key_states, value_states)
        n = key_states.shape[-2]
        if self.length + n > self.capacity:
            raise RuntimeError(f"KV cache capacity {self.capacity} exceeded")
        self.k_buf[:, :, self.length:self.length + n].copy_(key_states)
        self.v_buf[:, :, self.length:self.length + n].copy_(value_states)
        self.length += n
        self.keys = self.k_buf[:, :, :self.length]
        self.values = self.v_buf[:, :, :self.length]
        return self.keys, self.values

    def get_seq_length(self) -> int:
        return self.length

    def get_max_cache_shape(self) -> int:
        return self.capacity

    def reset(self) -> None:
        self.length = 0
        if self.is_initialized:
            self.keys, self.values = self.k_buf[:, :, :0], self.v_buf[:, :, :0]


class PreallocatedKVCache(Cache):
    """transformers Cache of ``PreallocatedLayer`` (one per decoder layer)."""

    def __init__(self, num_layers: int, capacity: int):
        super().__init__(layers=[PreallocatedLayer(capacity) for _ in range(num_layers)])


def hf_model_over_tp(runner) -> tuple[Qwen3ForCausalLM, "PreallocatedKVCache"]:
    """The reference's model API over a one-rank ``tp.Qwen3TPRunner``'s state: an
    HF ``Qwen3ForCausalLM`` whose attention layers are ``Qwen3SparseKernelAttention``
    (the runner's BigBird layout in its sparse layers, dense elsewhere) with every
    parameter a view of the runner's weights (no copy), and a
    ``PreallocatedKVCache`` over the runner's KV cache at ``runner.length``. Decoding
    through it runs the hook path (HF modules, ``pattern.build`` per call) from
    the same prefilled cache."""
    from transformers.models.qwen3.modeling_qwen3 import Qwen3RotaryEmbedding

    if runner.w.world != 1:
        raise ValueError("needs a one-rank runner")
    A, w = runner.A, runner.w
    D, H, Hkv = A.head_dim, A.heads, A.kv_heads
    cfg = Qwen3Config(vocab_size=A.vocab, hidden_size=A.hidden, intermediate_size=A.intermediate,
                      num_hidden_layers=A.layers, num_attention_heads=H, num_key_value_heads=Hkv, head_dim=D,
                      rms_norm_eps=A.eps, rope_theta=A.rope_theta, tie_word_embeddings=A.tie_embeddings,
                      max_position_embeddings=runner.capacity)
    cfg._attn_implementation = register_attention_implementation()
    cfg.sparse_attention_pattern = "bigbird"
    cfg.sparse_attention_layer_layouts = [[list(runner.layout)] if li in runner.sparse else None
                                          for li in range(A.layers)]
    cfg.sparse_attention_dense_impl = "cuda_sm100"
    with torch.device("meta"):
        model = Qwen3ForCausalLM(cfg)
        for li, layer in enumerate(model.model.layers):
            layer.self_attn = Qwen3SparseKernelAttention(cfg, li)

    def put(mod, t):
        mod._parameters["weight"] = nn.Parameter(t, requires_grad=False)

    put(model.model.embed_tokens, w.embed)
    put(model.model.norm, w.final_norm)
    put(model.lm_head, w.lm_head)
    for layer, L in zip(model.model.layers, w.layers):
        a, m = layer.self_attn, layer.mlp
        put(a.q_proj, L["qkv"][: H * D])
        put(a.k_proj, L["qkv"][H * D:(H + Hkv) * D])
        put(a.v_proj, L["qkv"][(H + Hkv) * D:])
        put(a.o_proj, L["o"])
        put(a.q_norm, L["qn"])
        put(a.k_norm, L["kn"])
        inter = L["gu"].shape[0] // 2
        put(m.gate_proj, L["gu"][:inter])
        put(m.up_proj, L["gu"][inter:])
        put(m.down_proj, L["down"])
        put(layer.input_layernorm, L["ln1"])
        put(layer.post_attention_layernorm, L["ln2"])
    dev = w.embed.device
    model.model.rotary_emb = Qwen3RotaryEmbedding(cfg, device=dev)
    model.eval()
    cache = PreallocatedKVCache(A.layers, runner.capacity)
    for li, cl in enumerate(cache.layers):
        cl.dtype, cl.device = w.embed.dtype, dev
        cl.k_buf, cl.v_buf = runner.k_cache[li], runner.v_cache[li]
        cl.length = runner.length
        cl.keys, cl.values = cl.k_buf[:, :, :cl.length], cl.v_buf[:, :, :cl.length]
        cl.is_initialized = True
    return model, cache


__all__ = [
    "Qwen3SparseKernelAttention", "replace_qwen3_attention_with_sparse", "build_sparse_attention_from_dense",
    "Qwen3SparseKernelForCausalLM", "PreallocatedKVCache", "PreallocatedLayer", "build_layer_block_experiments",
    "normalize_group_sparsities", "normalize_layer_group_sparsities", "hf_model_over_tp",
]
