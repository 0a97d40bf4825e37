"""Peer-mapped device arena for the expert-parallel exchange.

One symmetric allocation per rank (``torch.distributed._symmetric_memory``:
cuMem-backed, mapped into every peer process over NVLink), carved by a
host-side bump allocator that every rank runs identically.  A region request
names the byte size *for every rank* (all ranks know all ranks' routing
counts), so each rank knows the address of every peer's region without any
extra exchange: ``region.ptrs[r]`` is rank r's region as mapped in this
process.  The arena is reset at the start of every training micro-step;
regions live until the next reset, which is what the backward pass needs.

When a request does not fit, every rank makes the same decision and moves to a
new, larger chunk (a collective rendezvous), so the exchange never drops a
token for lack of buffer space.

``barrier()`` is the device-side phase separator of the exchange: one tiny
kernel that signals every peer with a release store of the next epoch of a
device counter and waits (bounded) for every peer's signal; a timeout is
recorded in the device status word.  Regions can also be kept for the life of
the arena (``reset`` is then never called): the expert-parallel exchange's
device-computed layout uses slabs of a fixed worst-case size per layer.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist

from ..ops import _ext

ALIGN = 256
MAX_RANKS = 8


@dataclass
class Region:
    ptrs: list          # per-rank device addresses (ints) valid in this process
    nbytes: list        # per-rank sizes in bytes
    local: torch.Tensor  # this rank's bytes (uint8 view)

    def view(self, dtype: torch.dtype, *shape: int) -> torch.Tensor:
        n = 1
        for s in shape:
            n *= s
        es = torch.empty((), dtype=dtype).element_size()
        return self.local[:n * es].view(dtype).view(*shape)


class _Chunk:
    def __init__(self, group, device, nbytes: int):
        import torch.distributed._symmetric_memory as symm_mem
        self.nbytes = nbytes
        self.buf = symm_mem.empty(nbytes, dtype=torch.uint8, device=device)
        self.handle = symm_mem.rendezvous(self.buf, group=group.group_name)
        self.ptrs = [int(p) for p in self.handle.buffer_ptrs]
        self.used = [0] * len(self.ptrs)


def _enable_group(group):
    try:
        import torch.distributed._symmetric_memory as symm_mem
        if hasattr(symm_mem, "enable_symm_mem_for_group"):
            symm_mem.enable_symm_mem_for_group(group.group_name)
    except Exception:  # pragma: no cover - API differences across torch versions
        pass


class SymmArena:
    def __init__(self, group, device: torch.device, chunk_bytes: int):
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        if self.world > MAX_RANKS:
            raise ValueError(f"peer-memory expert parallelism supports at most {MAX_RANKS} ranks per group")
        self.device = device
        self.chunk_bytes = max(ALIGN, chunk_bytes)
        _enable_group(group)
        self.chunks: list[_Chunk] = []
        self.cur = 0
        # signal flags: MAX_RANKS uint32 per rank (slot s = last epoch signalled by rank s)
        self._sig = _Chunk(group, device, ALIGN)
        self._sig.buf.zero_()
        self.sig_ptrs = self._sig.ptrs
        self.epoch = 0
        # barrier epochs are counted on the device (so CUDA graphs can replay barriers)
        self.epoch_ctr = torch.zeros(1, dtype=torch.int32, device=device)
        self.peak = [0] * self.world
        torch.cuda.synchronize(device)
        dist.barrier(group)

    # ------------------------------------------------------------------
    def reset(self):
        for c in self.chunks:
            c.used = [0] * self.world
        self.cur = 0

    def alloc(self, nbytes_per_rank: list[int]) -> Region:
        sizes = [(int(n) + ALIGN - 1) // ALIGN * ALIGN for n in nbytes_per_rank]
        while True:
            if self.cur >= len(self.chunks):
                need = max(self.chunk_bytes, 2 * max(sizes), self.nbytes())   # geometric growth
                self.chunks.append(_Chunk(self.group, self.device, need))
            c = self.chunks[self.cur]
            if all(c.used[r] + sizes[r] <= c.nbytes for r in range(self.world)):
                break
            self.cur += 1
        offs = list(c.used)
        for r in range(self.world):
            c.used[r] += sizes[r]
            self.peak[r] = max(self.peak[r], sum(ch.used[r] for ch in self.chunks))
        me = self.rank
        local = c.buf[offs[me]:offs[me] + max(sizes[me], 0)]
        return Region([c.ptrs[r] + offs[r] for r in range(self.world)], sizes, local)

    def barrier(self):
        """Device-side barrier over the group on the current stream (bounded wait).  The epoch
        lives in a device counter that every rank advances alike, so the barrier can be captured
        in a CUDA graph and replayed."""
        self.epoch += 1
        _ext.load().ep_barrier_dev(self.sig_ptrs, self.rank, self.epoch_ctr)

    def nbytes(self) -> int:
        return sum(c.nbytes for c in self.chunks)
