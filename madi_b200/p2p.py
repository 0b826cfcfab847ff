"""Rank-to-rank all-gather over NVLink for the column-split vocab head
(include/madi_q8.h: madi_xchg_*), a drop-in for the decoder's `exchange(out, inp)`.

Each rank's library object owns one device buffer that every peer maps through CUDA
IPC; an all-gather is one kernel that stores this rank's rows into every rank's buffer,
raises a sequence flag there and waits (bounded) for every peer's flag.  The ranks
must sit on distinct GPUs of one node -- two ranks' waiting kernels must never share
a GPU -- so construction compares the ranks' GPU ids and refuses otherwise
(`PeerExchange.usable` lets a caller fall back to a collective library).
"""
import ctypes
from typing import Optional

import torch

from . import _lib


def _device_id(device: torch.device) -> str:
    """A unique id of a GPU (its UUID)."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    return str(torch.cuda.get_device_properties(idx).uuid)


class PeerExchange:
    """All-gather of up to `cap_bytes` per rank over peer memory.  Collective
    construction: every rank of `group` must build one, in the same order."""

    def __init__(self, world: int, rank: int, cap_bytes: int, device: torch.device, group=None):
        import torch.distributed as dist
        self.world, self.rank, self.group = world, rank, group
        self.cap = (int(cap_bytes) + 15) // 16 * 16
        self._x = ctypes.c_void_p()
        ids = [None] * world
        dist.all_gather_object(ids, _device_id(device), group=group)
        if len(set(ids)) != world:
            raise RuntimeError(f"peer exchange needs one GPU per rank; ranks share GPUs: {ids}")
        L = _lib.load()
        _lib.check(L.madi_xchg_create(world, rank, self.cap, ctypes.byref(self._x)), "madi_xchg_create")
        h = ctypes.create_string_buffer(64)
        _lib.check(L.madi_xchg_handle(self._x, h), "madi_xchg_handle")
        handles = [None] * world
        dist.all_gather_object(handles, h.raw, group=group)
        for r in range(world):
            if r != rank:
                _lib.check(L.madi_xchg_open(self._x, r, ctypes.create_string_buffer(handles[r], 64)),
                           "madi_xchg_open")
        dist.barrier(group=group)        # every rank mapped every buffer before the first call

    @staticmethod
    def usable(world: int, device: torch.device, group=None) -> bool:
        """True when the ranks of `group` sit on distinct GPUs (collective call)."""
        import torch.distributed as dist
        ids = [None] * world
        dist.all_gather_object(ids, _device_id(device), group=group)
        return len(set(ids)) == world

    def __call__(self, out: torch.Tensor, inp: torch.Tensor, stream=None) -> None:
        """out (world x inp's bytes, rank-major) <- every rank's inp."""
        nbytes = inp.numel() * inp.element_size()
        if out.numel() * out.element_size() != self.world * nbytes or not (inp.is_contiguous() and out.is_contiguous()):
            raise ValueError("out must hold world x inp's bytes; both contiguous")
        s = stream if stream is not None else torch.cuda.current_stream(inp.device)
        rc = _lib.load().madi_xchg_allgather(self._x, inp.data_ptr(), nbytes, out.data_ptr(),
                                             getattr(s, "cuda_stream", s))
        _lib.check(rc, "madi_xchg_allgather")

    def close(self, group=None) -> None:
        """Collective: every rank unmaps its peers' buffers, the ranks meet, then each
        frees its own (no buffer is freed while a peer still maps it)."""
        import torch.distributed as dist
        group = group if group is not None else self.group
        if self._x:
            torch.cuda.synchronize()
            _lib.load().madi_xchg_unmap(self._x)
            dist.barrier(group=group)
            _lib.load().madi_xchg_destroy(self._x)
            self._x = ctypes.c_void_p()
