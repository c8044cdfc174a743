"""One-shot all-reduce over NVLink peer memory for the tensor-parallel decode step.

A decode step all-reduces a 7 KB hidden vector twice per layer; a collective library spends
tens of microseconds per such call. ``PeerAllReduce`` maps one small buffer per rank into every
peer's address space (CUDA IPC, handles exchanged through the process group once) and runs
``fpx_allreduce_bf16``: each rank stores its input and a flag into every rank's buffer, waits
for the flags in its own buffer (bounded waits) and sums the ranks' copies there in rank
order, so every rank gets the same bits. The call's counter lives in device memory, so the
kernel can be captured in a CUDA graph and replayed.
"""

from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from ._capi import call, lib, ptr, stream


class PeerAllReduce:
    def __init__(self, group=None, device=None, max_elems: int = 1 << 15):
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.device = torch.device(device or "cuda")
        self.max_elems = max_elems
        nbytes = lib().fpx_ar_buffer_bytes(max_elems)
        base = ctypes.c_void_p()
        handle = (ctypes.c_char * 64)()
        with torch.cuda.device(self.device):
            call("fpx_ar_create", ctypes.c_size_t(nbytes), ctypes.byref(base), handle)
        self.base = base.value
        handles = [None] * self.world
        dist.all_gather_object(handles, bytes(handle), group=group)
        self.peers = []
        with torch.cuda.device(self.device):
            for r, h in enumerate(handles):
                if r == self.rank:
                    self.peers.append(self.base)
                    continue
                peer = ctypes.c_void_p()
                call("fpx_ar_open", (ctypes.c_char * 64).from_buffer_copy(h), ctypes.byref(peer))
                self.peers.append(peer.value)
        self._bases = (ctypes.c_void_p * self.world)(*self.peers)
        dist.barrier(group=group)  # every rank has mapped every buffer before the first call

    def all_reduce_(self, t: torch.Tensor) -> torch.Tensor:
        """In-place sum over the ranks of a contiguous bf16 tensor of at most max_elems values."""
        call("fpx_allreduce_bf16", ptr(t), t.numel(), self._bases, self.rank, self.world, self.max_elems,
             stream(self.device))
        return t

    def fits(self, t: torch.Tensor) -> bool:
        return (t.dtype == torch.bfloat16 and t.is_contiguous() and t.numel() <= self.max_elems
                and t.numel() % 8 == 0)

    def error(self) -> int:
        code = ctypes.c_int(0)
        call("fpx_ar_error", ctypes.c_void_p(self.base), ctypes.byref(code))
        return code.value

    def close(self):
        with torch.cuda.device(self.device):
            for r, p in enumerate(self.peers):
                if r != self.rank and p:
                    call("fpx_ar_close", ctypes.c_void_p(p))
            if self.base:
                call("fpx_ar_destroy", ctypes.c_void_p(self.base))
        self.peers, self.base = [], None
