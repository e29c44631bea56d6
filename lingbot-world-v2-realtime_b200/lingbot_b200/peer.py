"""Peer heap: one device buffer per rank of a node, mapped into every other rank through CUDA IPC.

Every rank allocates the same number of bytes and carves it in the same order, so a buffer is named by
its byte offset and rank p's copy of it lives at `peers[p] + offset`. The sequence-split exchange
kernels (lbq_share_stats_push / lbq_chunk_totals / lbq_share_push / lbq_peer_wait) store straight into
the other ranks' KV-cache replicas and exchange areas through these mappings (NVLink peer stores), in
place of the host-staged q/k/v exchange of lingbot/parallel/split_dit.py:366-445 (`self.xch`).
Only plain peer loads and stores are used: no multicast objects are created.
"""
from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from . import _lib

ALIGN = 256


def _round_up(x, m):
    return (x + m - 1) // m * m


def exchange_records(record, group=None):
    """Every rank's (IPC handle bytes, offset, heap bytes) in rank order, through one all_gather_object of
    the process group (the only collective of the split's set-up). All ranks must pass the same heap
    size; a rank that never joins makes the call fail with the process group's timeout, not hang."""
    world = dist.get_world_size(group)
    everyone = [None] * world
    dist.all_gather_object(everyone, record, group=group)
    for p, (_, _, n) in enumerate(everyone):
        if n != record[2]:
            raise ValueError(f"rank {p} allocated a {n}-byte heap, this rank {record[2]}")
    return everyone


class PeerHeap:
    """`nbytes` of device memory on this rank, mapped by every rank of `group` (all ranks pass the same
    size and carve identically). With one rank (or no process group) nothing is exported."""

    def __init__(self, nbytes, device, group=None):
        self.group = group
        initialized = dist.is_available() and dist.is_initialized()
        self.world = dist.get_world_size(group) if initialized else 1
        self.rank = dist.get_rank(group) if initialized else 0
        self.nbytes = _round_up(int(nbytes), 1 << 21)
        self.buf = torch.empty(self.nbytes, dtype=torch.uint8, device=device)
        self.top = 0
        self._opened = []
        ptrs = [0] * self.world
        ptrs[self.rank] = self.buf.data_ptr()
        if self.world > 1:
            handle = (ctypes.c_char * 64)()
            off = ctypes.c_uint64(0)
            _lib.call("lbq_peer_export", ctypes.c_void_p(self.buf.data_ptr()), handle, ctypes.byref(off))
            everyone = exchange_records((bytes(handle), off.value, self.nbytes), group)
            for p, (h, o, n) in enumerate(everyone):
                if p == self.rank:
                    continue
                base = ctypes.c_void_p()
                _lib.call("lbq_peer_open", ctypes.create_string_buffer(h, 64), ctypes.byref(base))
                self._opened.append(base.value)
                ptrs[p] = base.value + o
        # u64 addresses stored as int64 bits
        self.peer_ptrs = ptrs
        self.peers = torch.tensor([p - (1 << 64) if p >= 1 << 63 else p for p in ptrs], dtype=torch.int64,
                                  device=device)

    def carve(self, shape, dtype, zero=True):
        """The next `shape`/`dtype` tensor of the heap (256-byte aligned offset)."""
        numel = 1
        for s in shape:
            numel *= int(s)
        size = numel * torch.empty((), dtype=dtype).element_size()
        off = _round_up(self.top, ALIGN)
        if off + size > self.nbytes:
            raise MemoryError(f"peer heap of {self.nbytes} bytes cannot hold {size} more at offset {off}")
        self.top = off + size
        t = self.buf[off:off + size].view(dtype).view(*shape)
        if zero:
            t.zero_()
        return t

    def offset(self, t):
        """Byte offset of tensor `t` inside this heap (it must have been carved from it)."""
        off = t.data_ptr() - self.buf.data_ptr()
        if off < 0 or off + t.numel() * t.element_size() > self.nbytes:
            raise ValueError("tensor is not inside the peer heap")
        return off

    def close(self):
        """Unmap the other ranks' heaps (this rank's own buffer is freed with the object)."""
        for base in self._opened:
            _lib.call("lbq_peer_close", ctypes.c_void_p(base))
        self._opened = []
