"""Tensor-parallel Qwen3 runner on the CUDA kernels (one rank) against the
masked-dense fp32 oracle model: last-position logits after a chunked prefill and
after each greedy decode step.

Logits tolerance (bf16 model vs fp32 reference arithmetic): max-abs deviation
<= 5e-2 * max|reference logit| and mean-abs <= 1e-2 * max|reference logit|."""
from __future__ import annotations

import pytest
import torch

from oracle.qwen3_model import masked_dense_forward
from sparseattentioninfer_b200 import _capi, tp

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
MAX_REL, MEAN_REL = 5e-2, 1e-2


@pytest.mark.parametrize("layout,sparse_layers,T,chunk", [
    ((128, 2, 4, 3), None, 1536, 512),      # the config-5 layout, every layer sparse
    ((64, 2, 4, 2), [0], 1000, 256),         # the config-4 layout, layer 1 dense, ragged T
])
def test_tp1_runner_logits_vs_masked_dense(layout, sparse_layers, T, chunk):
    A = tp.Qwen3Arch(hidden=512, layers=2, heads=32, kv_heads=8, head_dim=128, intermediate=1024, vocab=2000)
    w = tp.Qwen3TPWeights(A, 0, 1, seed=7, device=DEV)
    steps = 6
    r = tp.Qwen3TPRunner(w, 2, T + steps, layout, sparse_layers=sparse_layers)
    tok = torch.randint(0, A.vocab, (2, T), generator=torch.Generator().manual_seed(3))
    got = [r.prefill(tok.to(DEV), chunk=chunk).cpu()]
    t = got[0].argmax(-1, keepdim=True)
    feed = [t]
    for _ in range(steps):
        t, lg = r.step(t.to(DEV), return_logits=True)
        got.append(lg.cpu())
        feed.append(t.cpu())
    torch.cuda.synchronize()
    cache = []
    ref = [masked_dense_forward(w, tok, layout, sparse_layers, cache)]
    for t in feed[:-1]:
        ref.append(masked_dense_forward(w, t.cpu(), layout, sparse_layers, cache))
    for i, (a, b) in enumerate(zip(got, ref)):
        scale = b.abs().max().item()
        err = (a - b).abs()
        assert err.max().item() <= MAX_REL * scale and err.mean().item() <= MEAN_REL * scale, \
            f"position {i}: max {err.max().item():.3e} mean {err.mean().item():.3e} scale {scale:.3e}"
    assert _capi.device_error() == 0


def test_graph_decode_matches_eager_across_block_boundary():
    """Graph-replayed decode (device-side position, key count and CSR buffers)
    gives the eager step's logits while the cache grows across a key block."""
    A = tp.Qwen3Arch(hidden=512, layers=2, heads=32, kv_heads=8, head_dim=128, intermediate=1024, vocab=2000)
    w = tp.Qwen3TPWeights(A, 0, 1, seed=9, device=DEV)
    T, steps = 1000, 40                       # positions 1000..1039 cross block 1024 (bs 64)
    tok = torch.randint(0, A.vocab, (2, T), generator=torch.Generator().manual_seed(4)).to(DEV)
    eager = tp.Qwen3TPRunner(w, 2, T + steps, (64, 2, 4, 2), sparse_layers=[0], n_split=4)
    graph = tp.Qwen3TPRunner(w, 2, T + steps, (64, 2, 4, 2), sparse_layers=[0], n_split=4)
    l0 = eager.prefill(tok, chunk=256)
    l1 = graph.prefill(tok, chunk=256)
    assert torch.equal(l0, l1)
    graph.capture_decode()
    # memory handed out after the capture must never be written by a replay
    probes = [torch.full((256,), 7, dtype=torch.long, device=DEV) for _ in range(64)]
    t = l0.argmax(-1, keepdim=True)
    g = graph.step_graph(t)
    for i in range(steps):
        t_next, le = eager.step(t, return_logits=True)
        lg = graph.graph_logits
        assert torch.allclose(le, lg, atol=1e-3, rtol=0), f"step {i}: {(le - lg).abs().max().item():.3e}"
        assert torch.equal(t_next, g)
        t = t_next
        if i + 1 < steps:
            g = graph.step_graph()
    assert graph.length == eager.length == T + steps
    assert all(bool((p == 7).all()) for p in probes)
    assert _capi.device_error() == 0
