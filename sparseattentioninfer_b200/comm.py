"""Tensor-parallel all-reduce over NVLink peer memory, fused with the residual
add and RMSNorm that follow it in the decoder layer (sa_allreduce.cu).

``NvlinkAllReduce`` owns, per rank, a two-slot data region and a flag region
allocated by the C library and mapped into every other rank through CUDA IPC
(handles exchanged once over the process group). A row-parallel GEMM writes
its partial result into ``buffer(slot, shape)`` and ``add_rms_norm(slot, ...)``
sums all ranks' partials into the residual stream and normalises it, in one
kernel. Slots must alternate between consecutive calls (the decoder layer's
o_proj and down_proj do). Messages larger than ``max_bytes`` per slot go
through NCCL instead (``fits``).
"""
from __future__ import annotations

import ctypes
from typing import Sequence

import torch

from . import _capi

_MAX_WORLD = 8
_HANDLE_BYTES = 64


class _DevArray:
    """A raw device pointer seen as a torch tensor (CUDA array interface)."""

    def __init__(self, ptr: int, shape: Sequence[int], typestr: str, device_index: int):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr, "data": (ptr, False),
                                         "version": 3, "strides": None}
        self.device_index = device_index


def _as_tensor(ptr: int, shape, dtype: torch.dtype, device: torch.device) -> torch.Tensor:
    if dtype == torch.bfloat16:
        t = torch.as_tensor(_DevArray(ptr, shape, "<i2", device.index), device=device)
        return t.view(torch.bfloat16)
    if dtype == torch.int32:
        return torch.as_tensor(_DevArray(ptr, shape, "<i4", device.index), device=device)
    raise TypeError(dtype)


class NvlinkAllReduce:
    def __init__(self, max_bytes: int, group=None, device: torch.device | None = None, max_ctas: int = 256):
        import torch.distributed as dist
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        if self.world > _MAX_WORLD:
            raise ValueError(f"at most {_MAX_WORLD} ranks")
        self.device = device if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.max_bytes = (int(max_bytes) + 255) // 256 * 256
        self.max_ctas = int(max_ctas)
        lib = _capi.load()
        self._lib = lib
        self._own = []
        self._opened = []
        with torch.cuda.device(self.device):
            data = ctypes.c_void_p()
            flags = ctypes.c_void_p()
            _capi.check(lib.sa_ar_alloc(2 * self.max_bytes, ctypes.byref(data)))
            self._own.append(data.value)
            _capi.check(lib.sa_ar_alloc(self.max_ctas * _MAX_WORLD * 4, ctypes.byref(flags)))
            self._own.append(flags.value)
            hd = (ctypes.c_uint8 * _HANDLE_BYTES)()
            hf = (ctypes.c_uint8 * _HANDLE_BYTES)()
            _capi.check(lib.sa_ar_ipc_handle(data, hd))
            _capi.check(lib.sa_ar_ipc_handle(flags, hf))
            mine = (bytes(hd), bytes(hf))
            allh: list = [None] * self.world
            dist.all_gather_object(allh, mine, group=group)
            self._peers = _capi.ArPeers()
            self._peers.rank, self._peers.world = self.rank, self.world
            for q in range(self.world):
                if q == self.rank:
                    self._peers.data[q], self._peers.flags[q] = data.value, flags.value
                    continue
                ptrs = []
                for h in allh[q]:
                    buf = (ctypes.c_uint8 * _HANDLE_BYTES).from_buffer_copy(h)
                    p = ctypes.c_void_p()
                    _capi.check(lib.sa_ar_ipc_open(buf, ctypes.byref(p)))
                    self._opened.append(p.value)
                    ptrs.append(p.value)
                self._peers.data[q], self._peers.flags[q] = ptrs
            self.epoch = torch.zeros(self.max_ctas, dtype=torch.int32, device=self.device)
            self._peers.epoch = self.epoch.data_ptr()
            self._peers.max_ctas = self.max_ctas
        self._data_ptr = data.value
        dist.barrier(group=group)

    def fits(self, numel: int) -> bool:
        return numel * 2 <= self.max_bytes

    def buffer(self, slot: int, shape) -> torch.Tensor:
        """This rank's slot ``slot`` (0 or 1) as a contiguous bf16 tensor of ``shape``."""
        n = 1
        for s in shape:
            n *= int(s)
        if not self.fits(n):
            raise ValueError(f"{n} elements exceed the {self.max_bytes}-byte slot")
        return _as_tensor(self._data_ptr + slot * self.max_bytes, tuple(shape), torch.bfloat16, self.device)

    def add_rms_norm(self, slot: int, x: torch.Tensor, weight: torch.Tensor, eps: float,
                     out: torch.Tensor | None = None) -> torch.Tensor:
        """x += sum over ranks of their ``buffer(slot)`` (same shape as x), then
        returns RMSNorm(x) * weight."""
        n = x.shape[-1]
        x2 = x.view(-1, n)
        if out is None:
            out = torch.empty_like(x)
        o2 = out.view(-1, n)
        if x.dtype != torch.bfloat16 or weight.dtype != torch.bfloat16:
            raise TypeError("bf16 tensors expected")
        _capi.check(self._lib.sa_allreduce_add_rms_norm(
            ctypes.byref(self._peers), slot * self.max_bytes, x2.data_ptr(), weight.data_ptr(), o2.data_ptr(),
            x2.shape[0], n, x2.stride(0), o2.stride(0), float(eps), torch.cuda.current_stream(x.device).cuda_stream))
        return out

    def reset(self) -> None:
        """Re-arm after a timed-out call (the device error word read SA_DEV_ERR_TIMEOUT).
        A timeout leaves this rank's epochs advanced and its flags published while
        a peer's are not, so later calls would pair different epochs. All ranks
        call reset() together: each zeroes its epoch counters and its flag region,
        between two barriers, before the next call."""
        import torch.distributed as dist
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        with torch.cuda.device(self.device):
            self.epoch.zero_()
            _as_tensor(self._own[1], (self.max_ctas * _MAX_WORLD,), torch.int32, self.device).zero_()
            torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)

    def close(self) -> None:
        """Unmap the peers' regions and free this rank's (all ranks call it together)."""
        import torch.distributed as dist
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        with torch.cuda.device(self.device):
            for p in self._opened:
                self._lib.sa_ar_ipc_close(ctypes.c_void_p(p))
            self._opened = []
            dist.barrier(group=self.group)
            for p in self._own:
                self._lib.sa_ar_free(ctypes.c_void_p(p))
            self._own = []


__all__ = ["NvlinkAllReduce"]
