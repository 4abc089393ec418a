"""Tensor-parallel Qwen3 over KV groups (the full-model configurations).

The reference runs Qwen3 through transformers on one device with the sparse
attention hook (sparse_llm/qwen3/integrations/modeling_sparse_qwen3.py:200-260) and has no
collective. Here the same decoder arithmetic is sharded Megatron-style over the
KV groups, one process per GPU:

* rank r of N owns KV heads [r*Hkv/N, (r+1)*Hkv/N) and their Hq/Hkv query heads;
  q/k/v projections are column-parallel over those heads, o_proj is
  row-parallel over the same heads;
* gate/up are column-parallel over an equal slice of the intermediate size,
  down_proj row-parallel over it;
* the two row-parallel outputs of each layer are summed across ranks with one
  all-reduce each (NCCL over NVLink on GPUs, gloo on CPU), then added to the
  residual; embeddings, norms and lm_head are replicated.

Attention runs on this package's kernels: the prefill kernel over the full
prompt's BigBird CSR (chunked prefill reads the CSR rows of its query blocks,
so chunking does not change the schedule) and the split-KV decode kernel over
the decode row. The CSR is compiled for all Hq heads (the reference's random
blocks depend on the global query-head index) and each rank keeps its rows.

Weights are drawn per full matrix from a seeded generator and then sliced, so
every world size holds the same model; linear weights N(0, std), norms 1.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Optional, Sequence

import torch
import torch.nn.functional as F


@dataclass(frozen=True)
class Qwen3Arch:
    hidden: int
    layers: int
    heads: int
    kv_heads: int
    head_dim: int
    intermediate: int
    vocab: int
    rope_theta: float = 1e6
    eps: float = 1e-6
    tie_embeddings: bool = False


QWEN3_4B = Qwen3Arch(2560, 36, 32, 8, 128, 9728, 151936, tie_embeddings=True)
QWEN3_8B = Qwen3Arch(4096, 36, 32, 8, 128, 12288, 151936)


def kv_group_shard(n_kv: int, rank: int, world: int) -> tuple[int, int]:
    """KV heads [lo, hi) owned by ``rank``; the groups split evenly (world | n_kv)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of world {world}")
    if n_kv % world:
        raise ValueError(f"{n_kv} KV groups do not split over {world} ranks")
    per = n_kv // world
    return rank * per, (rank + 1) * per


def even_shard(n: int, rank: int, world: int) -> tuple[int, int]:
    """Columns [lo, hi) of an evenly split dimension (world | n)."""
    if n % world:
        raise ValueError(f"dimension {n} does not split over {world} ranks")
    per = n // world
    return rank * per, (rank + 1) * per


def _draw(seed: int, idx: int, shape, std: float, device) -> torch.Tensor:
    g = torch.Generator(device=device).manual_seed(seed * 1_000_003 + idx)
    return torch.randn(*shape, generator=g, device=device, dtype=torch.float32).mul_(std)


class Qwen3TPWeights:
    """One rank's shard of a random-init Qwen3 (see the module docstring for the split).

    Matrix ``idx`` numbering for the seeded draws: 0 embed, 1 lm_head, then per
    layer l: 16*l + 2 (q), +3 (k), +4 (v), +5 (o), +6 (gate), +7 (up), +8 (down).
    """

    def __init__(self, arch: Qwen3Arch, rank: int = 0, world: int = 1, *, seed: int = 0, std: float = 0.02,
                 device="cuda", dtype=torch.bfloat16):
        self.arch, self.rank, self.world = arch, rank, world
        A = arch
        D, rep = A.head_dim, A.heads // A.kv_heads
        self.kv_lo, self.kv_hi = kv_group_shard(A.kv_heads, rank, world)
        self.q_lo, self.q_hi = self.kv_lo * rep, self.kv_hi * rep
        self.i_lo, self.i_hi = even_shard(A.intermediate, rank, world)
        self.hq, self.hkv = self.q_hi - self.q_lo, self.kv_hi - self.kv_lo
        cast = lambda t: t.to(dtype).contiguous()  # noqa: E731
        self.embed = cast(_draw(seed, 0, (A.vocab, A.hidden), std, device))
        self.lm_head = self.embed if A.tie_embeddings else cast(_draw(seed, 1, (A.vocab, A.hidden), std, device))
        ones = lambda n: torch.ones(n, device=device, dtype=dtype)  # noqa: E731
        self.final_norm = ones(A.hidden)
        self.layers = []
        for l in range(A.layers):
            b = 16 * l
            wq = _draw(seed, b + 2, (A.heads * D, A.hidden), std, device)[self.q_lo * D:self.q_hi * D]
            wk = _draw(seed, b + 3, (A.kv_heads * D, A.hidden), std, device)[self.kv_lo * D:self.kv_hi * D]
            wv = _draw(seed, b + 4, (A.kv_heads * D, A.hidden), std, device)[self.kv_lo * D:self.kv_hi * D]
            wo = _draw(seed, b + 5, (A.hidden, A.heads * D), std, device)[:, self.q_lo * D:self.q_hi * D]
            wg = _draw(seed, b + 6, (A.intermediate, A.hidden), std, device)[self.i_lo:self.i_hi]
            wu = _draw(seed, b + 7, (A.intermediate, A.hidden), std, device)[self.i_lo:self.i_hi]
            wd = _draw(seed, b + 8, (A.hidden, A.intermediate), std, device)[:, self.i_lo:self.i_hi]
            self.layers.append({
                "ln1": ones(A.hidden), "ln2": ones(A.hidden), "qn": ones(D), "kn": ones(D),
                "qkv": cast(torch.cat([wq, wk, wv], 0)), "o": cast(wo),
                "gu": cast(torch.cat([wg, wu], 0)), "down": cast(wd),
            })
            del wq, wk, wv, wo, wg, wu, wd


def all_reduce_(t: torch.Tensor, group=None) -> torch.Tensor:
    """Sum ``t`` in place over the tensor-parallel group (no-op on one rank)."""
    if torch.distributed.is_available() and torch.distributed.is_initialized() and \
            torch.distributed.get_world_size(group) > 1:
        torch.distributed.all_reduce(t, group=group)
    return t


def mlp_block(x: torch.Tensor, L: dict, eps: float, group=None) -> torch.Tensor:
    """x += down(silu(gate(h)) * up(h)), h = RMSNorm(x); the row-parallel down output
    is all-reduced before the residual add (modeling_qwen3 Qwen3MLP)."""
    h = F.rms_norm(x, (x.shape[-1],), L["ln2"], eps)
    gu = h @ L["gu"].t()
    inter = gu.shape[-1] // 2
    y = (F.silu(gu[..., :inter]) * gu[..., inter:]) @ L["down"].t()
    x += all_reduce_(y, group)
    return x


def o_proj_block(x: torch.Tensor, att: torch.Tensor, L: dict, group=None) -> torch.Tensor:
    """x += o_proj(att) with att [.., hq_local*D]; all-reduced before the residual add."""
    x += all_reduce_(att @ L["o"].t(), group)
    return x


def rope_tables(arch: Qwen3Arch, capacity: int, device, dtype=torch.bfloat16):
    D = arch.head_dim
    inv = 1.0 / arch.rope_theta ** (torch.arange(0, D, 2, device=device, dtype=torch.float32) / D)
    ang = torch.outer(torch.arange(capacity, device=device, dtype=torch.float32), inv)
    emb = torch.cat([ang, ang], -1)
    return emb.cos().to(dtype), emb.sin().to(dtype)


def _rotate(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    D = x.shape[-1]
    return x * cos + torch.cat([-x[..., D // 2:], x[..., : D // 2]], -1) * sin


class Qwen3TPRunner:
    """Prefill (chunked) and greedy decode for one rank's shard.

    ``layout`` is the BigBird layout (bs, global, window, random) used in every
    sparse layer (``sparse_layers`` selects them; None = all); other layers run
    dense causal attention on the same kernels over a dense CSR.
    """

    def __init__(self, weights: Qwen3TPWeights, batch: int, capacity: int, layout: Sequence[int],
                 *, sparse_layers: Optional[Sequence[int]] = None, group=None, n_split: Optional[int] = None,
                 kernels=None):
        self.w = weights
        if kernels is None:
            from . import ops as kernels
        # ``kernels`` supplies compile_bigbird / prefill_fwd / decode_fwd with the
        # signatures of this package's ops module (the default); tests on hosts
        # without a GPU pass a checker object here.
        self.ops = kernels
        A = weights.arch
        self.A, self.B, self.capacity = A, batch, capacity
        self.layout = tuple(int(x) for x in layout)
        self.bs = self.layout[0]
        self.sparse = set(range(A.layers)) if sparse_layers is None else set(sparse_layers)
        self.group = group
        self.n_split = n_split
        dev = weights.embed.device
        self.dtype = dt = weights.embed.dtype
        D = A.head_dim
        self.num_sms = torch.cuda.get_device_properties(dev).multi_processor_count if dev.type == "cuda" else 148
        # zero-initialised: decode reads whole 64-key stages of the cache
        self.k_cache = [torch.zeros(batch, weights.hkv, capacity, D, device=dev, dtype=dt) for _ in range(A.layers)]
        self.v_cache = [torch.zeros_like(t) for t in self.k_cache]
        self.cos, self.sin = rope_tables(A, capacity, dev, dt)
        self.length = 0
        self._csr = {}
        self._ws = None

    # -- CSR -----------------------------------------------------------------
    def _rows(self, pairs, offs):
        lo, hi = self.w.q_lo, self.w.q_hi
        return pairs[lo:hi].contiguous(), offs[lo:hi].contiguous()

    def prefill_csr(self, T: int, dense: bool):
        """Full-prompt (T, T) CSR for this rank's query heads (cached per T)."""
        ops = self.ops
        key = ("prefill", T, dense)
        if key not in self._csr:
            A, bs = self.A, self.bs
            lay = [(bs, 0, math.ceil(T / bs), 0)] if dense else [self.layout]
            self._csr[key] = self._rows(*ops.compile_bigbird(lay, A.heads, T, T, bs, device=self.w.embed.device))
        return self._csr[key]

    def decode_csr(self, T_k: int, dense: bool):
        """Decode row (T_q = 1) for T_k keys; depends on T_k only through its block."""
        ops = self.ops
        bs = self.bs
        key = ("decode", dense, (T_k - 1) // bs, math.ceil(T_k / bs))
        hit = self._csr.get(key)
        if hit is None:
            nkb = math.ceil(T_k / bs)
            lay = [(bs, 0, nkb, 0)] if dense else [self.layout]
            width = nkb if dense else sum(self.layout[1:])
            hit = self._rows(*ops.compile_bigbird(lay, self.A.heads, 1, T_k, bs, device=self.w.embed.device,
                                                  width=width))
            for k in [k for k in self._csr if k[0] == "decode" and k[1] == dense]:
                del self._csr[k]
            self._csr[key] = hit
        return hit

    # -- prefill -------------------------------------------------------------
    @torch.no_grad()
    def prefill(self, tokens: torch.Tensor, chunk: int = 4096) -> torch.Tensor:
        """Run the prompt [B, T] through all layers (filling the cache) and return the
        last position's logits [B, vocab] (fp32)."""
        ops = self.ops
        A, w = self.A, self.w
        B, T = tokens.shape
        if T > self.capacity:
            raise ValueError(f"prompt of {T} tokens exceeds the cache capacity {self.capacity}")
        if chunk % self.bs:
            raise ValueError("chunk must be a multiple of the block size")
        D, hq, hkv = A.head_dim, w.hq, w.hkv
        csr = {d: self.prefill_csr(T, d) for d in (False, True)
               if (not d and self.sparse) or (d and len(self.sparse) < A.layers)}
        x_last = None
        for c0 in range(0, T, chunk):
            c1 = min(T, c0 + chunk)
            C = c1 - c0
            qb0, qb1 = c0 // self.bs, math.ceil(c1 / self.bs)
            x = F.embedding(tokens[:, c0:c1], w.embed)  # [B, C, hidden]
            cos, sin = self.cos[c0:c1].unsqueeze(1), self.sin[c0:c1].unsqueeze(1)  # [C, 1, D]
            att = torch.empty(B, C, hq, D, device=x.device, dtype=self.dtype)
            chunk_offs = {d: offs[:, qb0:qb1 + 1].contiguous() for d, (_, offs) in csr.items()}
            for li, L in enumerate(w.layers):
                h = F.rms_norm(x, (A.hidden,), L["ln1"], A.eps)
                qkv = (h @ L["qkv"].t()).view(B, C, hq + 2 * hkv, D)
                q = _rotate(F.rms_norm(qkv[:, :, :hq], (D,), L["qn"], A.eps), cos, sin)
                k = _rotate(F.rms_norm(qkv[:, :, hq:hq + hkv], (D,), L["kn"], A.eps), cos, sin)
                self.k_cache[li][:, :, c0:c1].copy_(k.transpose(1, 2))
                self.v_cache[li][:, :, c0:c1].copy_(qkv[:, :, hq + hkv:].transpose(1, 2))
                dense = li not in self.sparse
                pairs = csr[dense][0]
                ops.prefill_fwd(q.transpose(1, 2), self.k_cache[li][:, :, :c1], self.v_cache[li][:, :, :c1],
                                pairs, chunk_offs[dense], self.bs, out=att.transpose(1, 2))
                o_proj_block(x, att.view(B, C, hq * D), L, self.group)
                mlp_block(x, L, A.eps, self.group)
            x_last = x[:, -1]
        self.length = T
        return self._logits(x_last)

    def _logits(self, x: torch.Tensor) -> torch.Tensor:
        h = F.rms_norm(x, (self.A.hidden,), self.w.final_norm, self.A.eps)
        return (h @ self.w.lm_head.t()).float()

    # -- decode --------------------------------------------------------------
    @torch.no_grad()
    def step(self, tok: torch.Tensor, return_logits: bool = False):
        """One greedy decode step for tokens [B, 1]; returns the next tokens [B, 1]."""
        ops = self.ops
        A, w = self.A, self.w
        B = tok.shape[0]
        D, hq, hkv = A.head_dim, w.hq, w.hkv
        pos = self.length
        if pos >= self.capacity:
            raise ValueError("KV cache full")
        T_k = pos + 1
        cos, sin = self.cos[pos], self.sin[pos]
        x = F.embedding(tok[:, 0], w.embed)  # [B, hidden]
        ns = self.n_split if self.n_split is not None else max(1, min(64, math.ceil(self.num_sms / max(1, B * hkv))))
        if self._ws is None or self._ws[0].numel() < B * hq * ns * D:
            self._ws = (torch.empty(B * hq * ns * D, device=x.device), torch.empty(B * hq * ns * 2, device=x.device))
        att = torch.empty(B, hq, 1, D, device=x.device, dtype=self.dtype)
        for li, L in enumerate(w.layers):
            h = F.rms_norm(x, (A.hidden,), L["ln1"], A.eps)
            qkv = (h @ L["qkv"].t()).view(B, hq + 2 * hkv, D)
            q = _rotate(F.rms_norm(qkv[:, :hq], (D,), L["qn"], A.eps), cos, sin)
            k = _rotate(F.rms_norm(qkv[:, hq:hq + hkv], (D,), L["kn"], A.eps), cos, sin)
            self.k_cache[li][:, :, pos].copy_(k)
            self.v_cache[li][:, :, pos].copy_(qkv[:, hq + hkv:])
            pairs, offs = self.decode_csr(T_k, li not in self.sparse)
            ops.decode_fwd(q.unsqueeze(2), self.k_cache[li][:, :, :T_k], self.v_cache[li][:, :, :T_k], pairs, offs,
                           self.bs, n_split=ns, out=att, workspace=self._ws)
            o_proj_block(x, att.view(B, hq * D), L, self.group)
            mlp_block(x, L, A.eps, self.group)
        self.length = T_k
        logits = self._logits(x)
        nxt = logits.argmax(-1, keepdim=True)
        return (nxt, logits) if return_logits else nxt


__all__ = ["Qwen3Arch", "QWEN3_4B", "QWEN3_8B", "kv_group_shard", "even_shard", "Qwen3TPWeights",
           "Qwen3TPRunner", "all_reduce_", "mlp_block", "o_proj_block", "rope_tables"]
