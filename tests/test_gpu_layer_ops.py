"""Decoder-layer step kernels (sa_layer_ops.cu) against plain PyTorch fp32
references of the same arithmetic. Tolerances: one bf16 rounding of O(1)
values (atol 2e-2, rtol 1e-2); the residual add is bit-exact (bf16(x + y))."""
from __future__ import annotations

import pytest
import torch

from sparseattentioninfer_b200 import _capi, ops, tp

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _ref_norm_rope(t, w, cos, sin, eps):
    D = t.shape[-1]
    t = t * torch.rsqrt(t.pow(2).mean(-1, keepdim=True) + eps) * w
    return t * cos + torch.cat([-t[..., D // 2:], t[..., : D // 2]], -1) * sin


@pytest.mark.parametrize("D,B,T,Hq,Hkv,pos,device_pos", [
    (128, 8, 1, 32, 8, 777, False), (128, 2, 37, 8, 2, 100, False), (64, 3, 5, 8, 8, 0, True),
    (128, 4, 1, 4, 1, 2047, True),
])
def test_qk_norm_rope_append(D, B, T, Hq, Hkv, pos, device_pos):
    g = torch.Generator(device=DEV).manual_seed(1)
    cap = 2048 + 64
    qkv = torch.randn(B, T, Hq + 2 * Hkv, D, generator=g, device=DEV).to(torch.bfloat16) * 3
    qw = (1 + 0.1 * torch.randn(D, generator=g, device=DEV)).to(torch.bfloat16)
    kw = (1 + 0.1 * torch.randn(D, generator=g, device=DEV)).to(torch.bfloat16)
    A = tp.Qwen3Arch(hidden=64, layers=1, heads=Hq, kv_heads=Hkv, head_dim=D, intermediate=64, vocab=8)
    cos, sin = tp.rope_tables(A, cap, DEV)
    kc = torch.zeros(B, Hkv, cap, D, device=DEV, dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    pd = torch.tensor([pos], dtype=torch.int32, device=DEV) if device_pos else None
    q = ops.qk_norm_rope_append(qkv, qw, kw, cos, sin, kc, vc, Hq=Hq, Hkv=Hkv, pos=0 if device_pos else pos,
                                pos_dev=pd, eps=1e-6)
    x = qkv.float()
    c = cos[pos:pos + T].float().view(1, T, 1, D)
    s = sin[pos:pos + T].float().view(1, T, 1, D)
    rq = _ref_norm_rope(x[:, :, :Hq], qw.float(), c, s, 1e-6).transpose(1, 2)
    rk = _ref_norm_rope(x[:, :, Hq:Hq + Hkv], kw.float(), c, s, 1e-6).transpose(1, 2)
    torch.testing.assert_close(q.float(), rq, atol=2e-2, rtol=1e-2)
    torch.testing.assert_close(kc[:, :, pos:pos + T].float(), rk, atol=2e-2, rtol=1e-2)
    assert torch.equal(vc[:, :, pos:pos + T], qkv[:, :, Hq + Hkv:].transpose(1, 2))
    assert kc[:, :, :pos].abs().sum() == 0 and kc[:, :, pos + T:].abs().sum() == 0
    assert _capi.device_error() == 0


def test_qk_norm_rope_append_rejects_out_of_range_positions():
    qkv = torch.zeros(1, 4, 3, 64, device=DEV, dtype=torch.bfloat16)
    w = torch.ones(64, device=DEV, dtype=torch.bfloat16)
    A = tp.Qwen3Arch(hidden=64, layers=1, heads=1, kv_heads=1, head_dim=64, intermediate=64, vocab=8)
    cos, sin = tp.rope_tables(A, 16, DEV)
    kc = torch.zeros(1, 1, 16, 64, device=DEV, dtype=torch.bfloat16)
    with pytest.raises(_capi.SaError):
        ops.qk_norm_rope_append(qkv, w, w, cos, sin, kc, kc.clone(), Hq=1, Hkv=1, pos=13)


@pytest.mark.parametrize("rows,n,with_y", [(8, 4096, True), (4096, 2560, True), (3, 64, False)])
def test_add_rms_norm(rows, n, with_y):
    g = torch.Generator(device=DEV).manual_seed(2)
    x = torch.randn(rows, n, generator=g, device=DEV).to(torch.bfloat16)
    y = torch.randn(rows, n, generator=g, device=DEV).to(torch.bfloat16) if with_y else None
    w = (1 + 0.1 * torch.randn(n, generator=g, device=DEV)).to(torch.bfloat16)
    x0 = x.clone()
    out = ops.add_rms_norm(x, y, w, 1e-6)
    xs = (x0.float() + y.float()).to(torch.bfloat16) if with_y else x0
    assert torch.equal(x, xs)
    xf = xs.float()
    ref = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-6) * w.float()
    torch.testing.assert_close(out.float(), ref, atol=2e-2, rtol=1e-2)


@pytest.mark.parametrize("rows,inter", [(8, 12288), (1000, 9728), (1, 8)])
def test_silu_mul(rows, inter):
    g = torch.Generator(device=DEV).manual_seed(3)
    gu = (2 * torch.randn(rows, 2 * inter, generator=g, device=DEV)).to(torch.bfloat16)
    out = ops.silu_mul(gu)
    f = gu.float()
    ref = torch.nn.functional.silu(f[:, :inter]) * f[:, inter:]
    torch.testing.assert_close(out.float(), ref, atol=2e-2, rtol=1e-2)


@pytest.mark.parametrize("M,K,N,x_pad", [
    (8, 4096, 768, 0), (8, 512, 4096, 0), (8, 1536, 4096, 0), (1, 256, 16, 0), (3, 4096, 6144, 8),
    (5, 12288, 4096, 0), (8, 2560, 2560, 16), (7, 9728, 2560, 0),
])
def test_linear_m8(M, K, N, x_pad):
    """sa_linear_m8 against an fp32 matmul of the same bf16 operands (one bf16
    rounding of the output; K up to 12288 at N(0, 0.02) weights)."""
    g = torch.Generator(device=DEV).manual_seed(K + N + M)
    xs = torch.randn(M, K + x_pad, generator=g, device=DEV).to(torch.bfloat16)
    x = xs[:, :K]
    w = (0.02 * torch.randn(N, K, generator=g, device=DEV)).to(torch.bfloat16)
    ref = x.float() @ w.float().t()
    got = ops.linear_m8(x, w)
    assert got.shape == (M, N)
    err = (got.float() - ref).abs().max().item()
    assert err <= 1e-2 * ref.abs().max().item() + 1e-3, err
    # into a strided output (a view of a wider buffer)
    wide = torch.zeros(M, N + 32, device=DEV, dtype=torch.bfloat16)
    ops.linear_m8(x, w, out=wide[:, 16:16 + N])
    assert torch.equal(wide[:, 16:16 + N], got) and bool((wide[:, :16] == 0).all())
    assert _capi.device_error() == 0


@pytest.mark.parametrize("M,K,inter", [(8, 4096, 1536), (8, 4096, 12288), (2, 2560, 9728)])
def test_linear_m8_glu(M, K, inter):
    """Fused gate/up projection + SwiGLU == silu_mul of the two bf16 projections."""
    g = torch.Generator(device=DEV).manual_seed(inter)
    x = torch.randn(M, 1, K, generator=g, device=DEV).to(torch.bfloat16)
    w = (0.02 * torch.randn(2 * inter, K, generator=g, device=DEV)).to(torch.bfloat16)
    gu = (x.float() @ w.float().t()).to(torch.bfloat16)
    ref = torch.nn.functional.silu(gu[..., :inter].float()) * gu[..., inter:].float()
    got = ops.linear_m8(x, w, glu=True)
    assert got.shape == (M, 1, inter)
    err = (got.float() - ref).abs().max().item()
    assert err <= 2e-2 * ref.abs().max().item() + 1e-3, err
    assert _capi.device_error() == 0


def test_linear_m8_rejects_unsupported_shapes():
    x = torch.zeros(9, 256, device=DEV, dtype=torch.bfloat16)
    w = torch.zeros(16, 256, device=DEV, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="tokens"):
        ops.linear_m8(x, w)
    with pytest.raises(RuntimeError, match="multiple"):
        ops.linear_m8(x[:8, :200], w[:, :200])
