"""Seeded synthetic inputs of the benchmark configurations (shapes, patterns, values).

The reference measures on random tensors (sparse_attention_bench/config.py:49-61
``make_qkv``: torch.randn); these helpers fix the seeds and draw orders so the
CUDA path, the tests and the CPU baseline see identical inputs.

* CONFIG1  BigBird layer, B=1 H=8 S=1024 D=64, block 64, layout (64, 2, 3, 2).
* CONFIG2  arbitrary block mask, B=4 H=32 S=8192 D=128 bf16, block 128, every
           causal block kept with p=0.25 (diagonal always), seed 0.
* CONFIG3  GQA Qwen3-4B shape, B=2 Hq=32 Hkv=8 S=16384 D=128 bf16, block 64,
           per-KV-group BigBird layouts drawn from seed 2; q/k RMSNorm + RoPE.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch


@dataclass(frozen=True)
class LayerConfig:
    name: str
    B: int
    Hq: int
    Hkv: int
    S: int
    D: int
    block_size: int
    dtype: torch.dtype


CONFIG1 = LayerConfig("bigbird_layer_b1_h8_s1024_d64", 1, 8, 8, 1024, 64, 64, torch.float32)
CONFIG2 = LayerConfig("arbitrary_block_mask_b4_h32_s8192_d128", 4, 32, 32, 8192, 128, 128, torch.bfloat16)
CONFIG3 = LayerConfig("gqa_qwen3_4b_b2_h32kv8_s16384_d128", 2, 32, 8, 16384, 128, 64, torch.bfloat16)

CONFIG1_LAYOUT = (64, 2, 3, 2)


def seeded_qkv(seed: int, B: int, H: int, Hkv: int, T_q: int, T_k: int, D: int, *, device="cpu",
               dtype=torch.float32):
    """N(0,1) q, k, v drawn in that order from torch.Generator(device).manual_seed(seed)."""
    g = torch.Generator(device=device).manual_seed(seed)
    q = torch.randn(B, H, T_q, D, generator=g, device=device, dtype=torch.float32)
    k = torch.randn(B, Hkv, T_k, D, generator=g, device=device, dtype=torch.float32)
    v = torch.randn(B, Hkv, T_k, D, generator=g, device=device, dtype=torch.float32)
    return q.to(dtype), k.to(dtype), v.to(dtype)


def bernoulli_block_bitmap(H: int, nqb: int, nkb: int, p: float, seed: int, device="cpu") -> torch.Tensor:
    """Each causal block (kb <= qb) kept with probability p, the diagonal always.
    One torch.rand(H, nqb, nkb) draw from torch.Generator(device).manual_seed(seed)."""
    g = torch.Generator(device=device).manual_seed(seed)
    u = torch.rand(H, nqb, nkb, generator=g, device=device)
    qb = torch.arange(nqb, device=device).view(1, -1, 1)
    kb = torch.arange(nkb, device=device).view(1, 1, -1)
    keep = ((u < p) & (kb <= qb)) | (kb == qb)
    return keep.to(torch.uint8)


def config3_group_layouts(seed: int = 2, n_groups: int = 8, block_size: int = 64):
    """Per KV group, in group order, draws window in [2, 8], global in [1, 4],
    random in [0, 3] (torch.randint, that order) from torch.Generator().manual_seed(seed).
    Returns ((bs, global, window, random), ...) — the reference's layout tuple order."""
    g = torch.Generator().manual_seed(seed)
    out = []
    for _ in range(n_groups):
        w = int(torch.randint(2, 9, (1,), generator=g))
        gl = int(torch.randint(1, 5, (1,), generator=g))
        r = int(torch.randint(0, 4, (1,), generator=g))
        out.append((block_size, gl, w, r))
    return tuple(out)


def rms_norm(x: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    """Qwen3RMSNorm with unit weight, computed in fp32."""
    xf = x.float()
    return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)).to(x.dtype)


def rope(x: torch.Tensor, theta: float = 1e6, offset: int = 0) -> torch.Tensor:
    """Rotate-half RoPE (transformers apply_rotary_pos_emb convention) over [.., T, D]."""
    T, D = x.shape[-2], x.shape[-1]
    inv = 1.0 / (theta ** (torch.arange(0, D, 2, device=x.device, dtype=torch.float32) / D))
    pos = torch.arange(offset, offset + T, device=x.device, dtype=torch.float32)
    ang = torch.outer(pos, inv)
    emb = torch.cat([ang, ang], dim=-1)
    cos, sin = emb.cos(), emb.sin()
    xf = x.float()
    x1, x2 = xf[..., : D // 2], xf[..., D // 2:]
    rot = torch.cat([-x2, x1], dim=-1)
    return (xf * cos + rot * sin).to(x.dtype)


def retained_flops(offsets: torch.Tensor, pairs: torch.Tensor, B: int, bs: int, D: int) -> int:
    """4 * bs^2 * D per retained (b, q-head, q-block, k-block) entry (QK^T + PV,
    sparse_attention_bench/metrics/flops.py:23-32 per kept block pair)."""
    nnz = int(offsets[:, -1].long().sum().item())
    return 4 * bs * bs * D * nnz * B


def nkb(T: int, bs: int) -> int:
    return math.ceil(T / bs)
