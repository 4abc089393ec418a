"""Timeout and re-arm of the fused NVLink all-reduce on one GPU, with no peer
process: rank 0 of a two-rank set whose "peer 1" regions are plain buffers on
the same device that nothing ever writes. The bounded wait for peer 1's flag
runs out (2 s), the call leaves x unchanged and the device error word reads
SA_DEV_ERR_TIMEOUT; after the reset (epochs and flags zeroed, what
NvlinkAllReduce.reset() does on every rank) a one-rank call computes
x += y, out = RMSNorm(x) * w and advances the epochs from zero again."""
from __future__ import annotations

import ctypes

import pytest
import torch

from sparseattentioninfer_b200 import _capi

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
SA_DEV_ERR_TIMEOUT = 1
MAX_CTAS = 64


def _peers(world, data, flags, epoch):
    p = _capi.ArPeers()
    p.rank, p.world = 0, world
    for q in range(world):
        p.data[q], p.flags[q] = data[q].data_ptr(), flags[q].data_ptr()
    p.epoch = epoch.data_ptr()
    p.max_ctas = MAX_CTAS
    return p


def test_timeout_leaves_x_then_reset_rearms():
    lib = _capi.load()
    assert _capi.device_error() == 0
    rows, n = 4, 512
    g = torch.Generator(device=DEV).manual_seed(1)
    data = [torch.randn(2, rows, n, device=DEV, generator=g).to(torch.bfloat16) for _ in range(2)]
    flags = [torch.zeros(MAX_CTAS * 8, dtype=torch.int32, device=DEV) for _ in range(2)]
    epoch = torch.zeros(MAX_CTAS, dtype=torch.int32, device=DEV)
    x0 = torch.randn(rows, n, device=DEV, generator=g).to(torch.bfloat16)
    w = torch.randn(n, device=DEV, generator=g).to(torch.bfloat16)
    x, out = x0.clone(), torch.empty_like(x0)
    stream = torch.cuda.current_stream().cuda_stream

    def call(world):
        p = _peers(world, data, flags, epoch)
        _capi.check(lib.sa_allreduce_add_rms_norm(ctypes.byref(p), 0, x.data_ptr(), w.data_ptr(), out.data_ptr(),
                                                  rows, n, n, n, 1e-6, stream))
        torch.cuda.synchronize()

    call(2)  # peer 1 never arrives
    assert _capi.device_error() == SA_DEV_ERR_TIMEOUT
    assert torch.equal(x, x0)
    assert int(epoch.max()) >= 1 and int(flags[1].max()) >= 1   # advanced / published: out of step
    epoch.zero_()
    for f in flags:
        f.zero_()
    call(1)
    assert _capi.device_error() == 0
    ref_x = (x0.float() + data[0][0].float()).to(torch.bfloat16)
    assert torch.equal(x, ref_x)
    xf = ref_x.float()
    ref_out = (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-6) * w.float()).to(torch.bfloat16)
    assert (out.float() - ref_out.float()).abs().max().item() <= 2e-2
    assert int(epoch.max()) == 1
