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


def rope_tables(arch: Qwen3Arch, capacity: int, device, dtype=torch.bfloat16):
    D = arch.head_dim
    inv = 1.0 / arch.rope_theta ** (torch.arange(0, D, 2, device=device, dtype=torch.float32) / D)
    ang = torch.outer(torch.arange(capacity, device=device, dtype=torch.float32), inv)
    emb = torch.cat([ang, ang], -1)
    return emb.cos().to(dtype), emb.sin().to(dtype)


class Qwen3TPRunner:
    """Prefill (chunked) and greedy decode for one rank's shard.

    ``layout`` is the BigBird layout (bs, global, window, random) used in every
    sparse layer (``sparse_layers`` selects them; None = all); other layers run
    dense causal attention on the same kernels over a dense CSR.
    """

    def __init__(self, weights: Qwen3TPWeights, batch: int, capacity: int, layout: Sequence[int],
                 *, sparse_layers: Optional[Sequence[int]] = None, group=None, n_split: Optional[int] = None,
                 kernels=None, comm=None, dense_impl: str = "cuda_sm100",
                 overlap_prefill: bool = True, skinny_linear: bool = True):
        self.w = weights
        # ``skinny_linear``: steps of at most 8 tokens (decode at batch <= 8) run
        # their four projections through ops.linear_m8 (a weight-streaming
        # kernel, SwiGLU fused into gate/up) instead of cuBLAS GEMMs.
        self.skinny_linear = skinny_linear
        # dense layers: "cuda_sm100" (this package's kernels over a dense CSR;
        # graph-capturable) or "sdpa" (PyTorch SDPA, the library comparator; eager
        # decode only, its causal mask is top-left aligned so prefill stays on
        # the package's kernel)
        if dense_impl not in ("cuda_sm100", "sdpa"):
            raise ValueError(dense_impl)
        self.dense_impl = dense_impl
        # ``comm`` (comm.NvlinkAllReduce): messages that fit its slots take the
        # fused NVLink all-reduce + add + RMSNorm kernel instead of NCCL.
        self.comm = comm
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
        self._comm_stream = None
        self.overlap_prefill = overlap_prefill
        self._graph = None
        self._g_csr = {}

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

    # -- one decoder layer ------------------------------------------------------
    def _layer(self, x: torch.Tensor, h: torch.Tensor, li: int, *, T: int, pos: int, pos_dev, attend,
               next_norm: torch.Tensor) -> torch.Tensor:
        """Layer ``li`` on the residual stream x [B, T, hidden] whose RMSNorm(ln1) is
        h: q/k/v projection, fused q/k norm + RoPE + cache append at positions
        pos.. (``pos_dev`` on the device), ``attend(li, q) -> att [B, T, hq*D]``,
        o_proj + all-reduce + residual add + ln2, SwiGLU MLP + all-reduce +
        residual add, and the next RMSNorm (``next_norm``); returns that."""
        ops, A, w = self.ops, self.A, self.w
        L = w.layers[li]
        B = x.shape[0]
        D, hq, hkv = A.head_dim, w.hq, w.hkv
        skinny = self.skinny_linear and B * T <= 8

        def proj(inp, name, out=None, glu=False):
            if skinny:
                return ops.linear_m8(inp, L[name], out=out, glu=glu)
            y = torch.matmul(inp, L[name].t(), out=out)
            return ops.silu_mul(y) if glu else y

        qkv = proj(h, "qkv").view(B, T, hq + 2 * hkv, D)
        q = ops.qk_norm_rope_append(qkv, L["qn"], L["kn"], self.cos, self.sin, self.k_cache[li], self.v_cache[li],
                                    Hq=hq, Hkv=hkv, pos=pos, pos_dev=pos_dev, eps=A.eps)
        att = attend(li, q)
        if self.comm is not None and self.comm.fits(B * T * A.hidden):
            shape = (B, T, A.hidden)
            proj(att, "o", out=self.comm.buffer(0, shape))
            h = self.comm.add_rms_norm(0, x, L["ln2"], A.eps)
            act = proj(h, "gu", glu=True)
            proj(act, "down", out=self.comm.buffer(1, shape))
            return self.comm.add_rms_norm(1, x, next_norm, A.eps)
        h = ops.add_rms_norm(x, all_reduce_(proj(att, "o"), self.group), L["ln2"], A.eps)
        act = proj(h, "gu", glu=True)
        return ops.add_rms_norm(x, all_reduce_(proj(act, "down"), self.group), next_norm, A.eps)

    def _forward(self, tok: torch.Tensor, pos: int, pos_dev, attend) -> torch.Tensor:
        """All layers for tokens [B, T] at positions pos..; returns the final-norm
        hidden state of the last position [B, hidden]."""
        A, w = self.A, self.w
        B, T = tok.shape
        x = F.embedding(tok, w.embed)  # [B, T, hidden]
        h = self.ops.add_rms_norm(x, None, w.layers[0]["ln1"], A.eps)
        for li in range(A.layers):
            nxt = w.layers[li + 1]["ln1"] if li + 1 < A.layers else w.final_norm
            h = self._layer(x, h, li, T=T, pos=pos, pos_dev=pos_dev, attend=attend, next_norm=nxt)
        return h[:, -1]

    def _half_stream(self, tok: torch.Tensor, b0: int, b1: int, pos: int, attend, out: list):
        """The decoder layers for batch rows [b0, b1) as a generator that yields each
        row-parallel partial sum (o_proj, then down_proj, per layer) for the caller
        to all-reduce in place before resuming it; leaves the last position's
        final-norm hidden state in ``out``."""
        ops, A, w = self.ops, self.A, self.w
        D, hq, hkv = A.head_dim, w.hq, w.hkv
        B, T = b1 - b0, tok.shape[1]
        x = F.embedding(tok[b0:b1], w.embed)
        h = ops.add_rms_norm(x, None, w.layers[0]["ln1"], A.eps)
        for li in range(A.layers):
            L = w.layers[li]
            qkv = (h @ L["qkv"].t()).view(B, T, hq + 2 * hkv, D)
            q = ops.qk_norm_rope_append(qkv, L["qn"], L["kn"], self.cos, self.sin, self.k_cache[li][b0:b1],
                                        self.v_cache[li][b0:b1], Hq=hq, Hkv=hkv, pos=pos, eps=A.eps)
            y = attend(li, q, b0, b1) @ L["o"].t()
            yield y
            h = ops.add_rms_norm(x, y, L["ln2"], A.eps)
            y = ops.silu_mul(h @ L["gu"].t()) @ L["down"].t()
            yield y
            nxt = w.layers[li + 1]["ln1"] if li + 1 < A.layers else w.final_norm
            h = ops.add_rms_norm(x, y, nxt, A.eps)
        out.append(h[:, -1])

    def _forward_overlapped(self, tok: torch.Tensor, pos: int, attend) -> torch.Tensor:
        """_forward with the NCCL all-reduces hidden behind compute: the batch is
        split in two halves whose layers are interleaved on the compute stream,
        while a second stream all-reduces one half's partial sum as the other half
        computes (the halves share nothing until the logits). Same arithmetic
        per row as _forward."""
        B = tok.shape[0]
        halves = [(0, B // 2), (B // 2, B)]
        outs = [[], []]
        gens = [self._half_stream(tok, b0, b1, pos, attend, outs[i]) for i, (b0, b1) in enumerate(halves)]
        cuda = tok.is_cuda  # on the host (gloo ranks) the same interleaving runs in order
        comp = torch.cuda.current_stream(tok.device) if cuda else None
        comm = self._comm_stream
        if cuda and (comm is None or comm.device != tok.device):
            comm = self._comm_stream = torch.cuda.Stream(device=tok.device)
        ev_ar = [None, None]

        def launch(i, y):
            if not cuda:
                all_reduce_(y, self.group)
                return
            ev = torch.cuda.Event()
            ev.record(comp)
            with torch.cuda.stream(comm):
                comm.wait_event(ev)
                all_reduce_(y, self.group)
                y.record_stream(comm)
                done = torch.cuda.Event()
                done.record(comm)
            ev_ar[i] = done

        active = [True, True]
        for i in range(2):
            launch(i, next(gens[i]))
        while any(active):
            for i in range(2):
                if not active[i]:
                    continue
                if cuda:
                    comp.wait_event(ev_ar[i])
                try:
                    y = gens[i].send(None)
                except StopIteration:
                    active[i] = False
                    continue
                launch(i, y)
        return torch.cat([outs[0][0], outs[1][0]], 0)

    def _logits(self, h_last: torch.Tensor) -> torch.Tensor:
        return (h_last @ self.w.lm_head.t()).float()

    # -- prefill ---------------------------------------------------------------
    @torch.no_grad()
    def prefill(self, tokens: torch.Tensor, chunk: int = 4096) -> torch.Tensor:
        """Run the prompt [B, T] through all layers (filling the cache) and return the
        last position's logits [B, vocab] (fp32). Chunks of ``chunk`` positions attend
        through the CSR rows of their query blocks in the full prompt's CSR."""
        ops = self.ops
        A, w = self.A, self.w
        B, T = tokens.shape
        if T > self.capacity:
            raise ValueError(f"prompt of {T} tokens exceeds the cache capacity {self.capacity}")
        if chunk % self.bs:
            raise ValueError("chunk must be a multiple of the block size")
        D, hq = A.head_dim, w.hq
        csr = {d: self.prefill_csr(T, d) for d in (False, True)
               if (not d and self.sparse) or (d and len(self.sparse) < A.layers)}
        h_last = None
        for c0 in range(0, T, chunk):
            c1 = min(T, c0 + chunk)
            C = c1 - c0
            qb0, qb1 = c0 // self.bs, math.ceil(c1 / self.bs)
            att = torch.empty(B, C, hq, D, device=tokens.device, dtype=self.dtype)
            chunk_offs = {d: offs[:, qb0:qb1 + 1].contiguous() for d, (_, offs) in csr.items()}

            def attend(li, q, b0=0, b1=B, c1=c1, att=att, chunk_offs=chunk_offs):
                dense = li not in self.sparse
                a = att[b0:b1]
                ops.prefill_fwd(q, self.k_cache[li][b0:b1, :, :c1], self.v_cache[li][b0:b1, :, :c1],
                                csr[dense][0], chunk_offs[dense], self.bs, out=a.transpose(1, 2))
                return a.view(b1 - b0, -1, hq * D)

            if self._overlap_prefill(B):
                h_last = self._forward_overlapped(tokens[:, c0:c1], c0, attend)
            else:
                h_last = self._forward(tokens[:, c0:c1], c0, None, attend)
        self.length = T
        return self._logits(h_last)

    def _overlap_prefill(self, B: int) -> bool:
        """Prefill all-reduces overlap compute (two batch halves) on more than one
        rank with an even batch; ``overlap_prefill=False`` turns it off."""
        if not self.overlap_prefill or B < 2 or B % 2:
            return False
        import torch.distributed as dist
        return dist.is_available() and dist.is_initialized() and dist.get_world_size(self.group) > 1

    # -- decode ----------------------------------------------------------------
    def _n_split(self) -> int:
        if self.n_split is not None:
            return self.n_split
        return max(1, min(64, math.ceil(self.num_sms / max(1, self.B * self.w.hkv))))

    def _workspace(self, ns: int, device):
        B, hq, D = self.B, self.w.hq, self.A.head_dim
        if self._ws is None or self._ws[0].numel() < B * hq * ns * D:
            self._ws = (torch.empty(B * hq * ns * D, device=device), torch.empty(B * hq * ns * 2, device=device))
        return self._ws

    @torch.no_grad()
    def step(self, tok: torch.Tensor, return_logits: bool = False):
        """One greedy decode step for tokens [B, 1]; returns the next tokens [B, 1]."""
        ops = self.ops
        A, w = self.A, self.w
        B = tok.shape[0]
        pos = self.length
        if pos >= self.capacity:
            raise ValueError("KV cache full")
        T_k = pos + 1
        ns = self._n_split()
        ws = self._workspace(ns, tok.device)
        att = torch.empty(B, w.hq, 1, A.head_dim, device=tok.device, dtype=self.dtype)

        def attend(li, q):
            kc, vc = self.k_cache[li][:, :, :T_k], self.v_cache[li][:, :, :T_k]
            if li not in self.sparse and self.dense_impl == "sdpa":
                return F.scaled_dot_product_attention(q, kc, vc, enable_gqa=True).view(B, 1, -1)
            pairs, offs = self.decode_csr(T_k, li not in self.sparse)
            ops.decode_fwd(q, kc, vc, pairs, offs, self.bs, n_split=ns, out=att, workspace=ws)
            return att.view(B, 1, -1)

        logits = self._logits(self._forward(tok, pos, None, attend))
        self.length = T_k
        nxt = logits.argmax(-1, keepdim=True)
        return (nxt, logits) if return_logits else nxt

    # -- graph-captured decode ---------------------------------------------------
    @torch.no_grad()
    def capture_decode(self) -> None:
        """Record one decode step (all layers, logits, argmax, position advance) in
        a CUDA graph. The step reads its position and key count from device
        counters and recomputes its decode CSR rows on the device from the key
        count (ops.bigbird_decode_row), so replays need no host work."""
        if self.dense_impl == "sdpa" and len(self.sparse) < self.A.layers:
            raise RuntimeError("dense_impl='sdpa' cannot be captured (its length is a host value)")
        ops = self.ops
        A, w = self.A, self.w
        dev = w.embed.device
        B, D = self.B, A.head_dim
        ns = self._n_split()
        ws = self._workspace(ns, dev)
        nkb_cap = math.ceil(self.capacity / self.bs)
        self._g_csr = {}
        for dense in (False, True):
            if (not dense and self.sparse) or (dense and len(self.sparse) < A.layers):
                width = nkb_cap if dense else sum(self.layout[1:])
                self._g_csr[dense] = (torch.zeros(w.hq, width, dtype=torch.int32, device=dev),
                                      torch.zeros(w.hq, 2, dtype=torch.int32, device=dev))
        self._g_tok = torch.zeros(B, 1, dtype=torch.long, device=dev)
        self._g_pos = torch.zeros(1, dtype=torch.int32, device=dev)   # position of the fed token
        self._g_len = torch.zeros(1, dtype=torch.int32, device=dev)   # keys after the append
        att = torch.empty(B, w.hq, 1, D, device=dev, dtype=self.dtype)
        # The graph replays into these addresses and holds no reference to them:
        # the runner keeps every buffer the recorded step touches alive.
        self._g_keep = (att, ws)

        def attend(li, q):
            gp, go = self._g_csr[li not in self.sparse]
            ops.decode_fwd(q, self.k_cache[li], self.v_cache[li], gp, go, self.bs, n_split=ns, out=att,
                           workspace=ws, seq_len=self._g_len)
            return att.view(B, 1, -1)

        dense_layout = [(self.bs, 0, 1 << 30, 0)]  # window wider than any cache: every causal block

        def body():
            for dense, (gp, go) in self._g_csr.items():
                ops.bigbird_decode_row(dense_layout if dense else [self.layout], A.heads, self._g_len, self.bs, gp, go,
                                       head_lo=w.q_lo)
            logits = self._logits(self._forward(self._g_tok, 0, self._g_pos, attend))
            self._g_tok.copy_(logits.argmax(-1, keepdim=True))
            self._g_pos.add_(1)
            self._g_len.add_(1)
            return logits

        def rewind(p):
            self._g_pos.fill_(p)
            self._g_len.fill_(p + 1)

        # warm the body once on a side stream (allocator, library handles), then
        # rewind the counters and record
        saved = self.length
        rewind(saved)
        s = torch.cuda.Stream(device=dev)
        s.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(s):
            body()
        torch.cuda.current_stream(dev).wait_stream(s)
        rewind(saved)
        self._graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self._graph, capture_error_mode="thread_local"):
            self._g_logits = body()
        rewind(saved)
        self._graph_len = saved

    @torch.no_grad()
    def step_graph(self, tok: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Replay the captured step. ``tok`` [B, 1] sets the fed token (needed on the
        first replay; default: the previous replay's argmax, kept on the device).
        Returns the device buffer holding the next tokens [B, 1] (overwritten by
        the next replay)."""
        if self._graph is None:
            raise RuntimeError("capture_decode() first")
        pos = self.length
        if pos >= self.capacity:
            raise ValueError("KV cache full")
        moved = pos != self._graph_len  # the host moved the cache (prefill / eager steps)
        if moved:
            self._g_pos.fill_(pos)
            self._g_len.fill_(pos + 1)
        if tok is not None:
            self._g_tok.copy_(tok)
        self._graph.replay()
        self.length = self._graph_len = pos + 1
        return self._g_tok

    @property
    def graph_logits(self) -> torch.Tensor:
        """Logits [B, vocab] of the last replay."""
        return self._g_logits


__all__ = ["Qwen3Arch", "QWEN3_4B", "QWEN3_8B", "kv_group_shard", "even_shard", "Qwen3TPWeights",
           "Qwen3TPRunner", "all_reduce_", "rope_tables"]
