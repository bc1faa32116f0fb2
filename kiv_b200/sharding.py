"""Exchanges of the sharded cold tier (one process per GPU of one box).

Two partitions exist.  Sequence sharding (``batch_group``): each rank holds
its own sequences of the batch; the only exchange is the page union, which
the reference takes across the whole batch (kiv/cold_store.py:224) -- the
ranks OR their coarse page marks (``all_or_bits``) before the fine pass, and
everything after it is per sequence.  Page sharding (``shard_group``) splits
one sequence's cold pages:

The cold tier of a layer is partitioned by page over the GPUs of one box (page
p lives on rank p % world), and every rank keeps every page's summary, so the
coarse pass is exact on each rank.  On CUDA the fine pass then exchanges the
candidates themselves: each rank scores its pages of the union and stores the
keys into every rank's exchange arena over NVLink, every rank takes the exact
global top-P (``kiv_fine_exchange_select``), and the attention reads each
selected row from its owner's cold tier through a CUDA IPC mapping
(``map_peers``, ``kiv_attend_peers``), so every rank computes the full output
with no further exchange.  Shapes outside those kernels (and the collective
transport) exchange lists instead -- per-batch-row fine candidates (score,
token), then per-row attention partials (out, max, sum) -- and every rank
merges them identically.

Every rank allocates an exchange arena, the ranks swap CUDA IPC handles once
over the process group, and the kernels store into the peers' arenas as words
that carry the exchange's flag and wait (bounded) until every rank's words
carry it.  ``all_gather`` / ``all_reduce_sum`` (the process group's
collectives) remain for the API paths that return tensors and for CPU process
groups.
"""

from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist


class ShardComm:
    """A ``torch.distributed`` process group plus the peer-memory exchange arenas."""

    def __init__(self, group=None) -> None:
        self.group = group
        self.rank = dist.get_rank(group)
        self.size = dist.get_world_size(group)
        self._arenas: dict = {}
        self._peer_maps: dict = {}
        self._peer_bases: dict = {}      # (rank, its allocation base) -> (mapped base, device)

    def exchange(self, nbytes: int, device: torch.device):
        """The exchange descriptor of arenas of ``nbytes`` (every rank calls this
        with the same size; the first call allocates and maps them collectively)."""
        from . import _native as nat

        key = (int(nbytes), device.index)
        hit = self._arenas.get(key)
        if hit is not None:
            return hit[0]
        if self.size > nat.MAX_PEERS:
            raise nat.KIVNativeError(f"peer exchange supports up to {nat.MAX_PEERS} ranks, got {self.size}")
        L = nat.lib()
        own = ctypes.c_void_p()
        handle = (ctypes.c_ubyte * nat.IPC_HANDLE_BYTES)()
        with torch.cuda.device(device):
            nat.check(L.kiv_peer_alloc(int(nbytes), ctypes.byref(own), handle), "peer_alloc")
            handles = [None] * self.size
            dist.all_gather_object(handles, bytes(handle), group=self.group)
            arenas, opened = [], []
            for r, hb in enumerate(handles):
                if r == self.rank:
                    arenas.append(own.value)
                    continue
                p = ctypes.c_void_p()
                buf = (ctypes.c_ubyte * nat.IPC_HANDLE_BYTES).from_buffer_copy(hb)
                nat.check(L.kiv_peer_open(buf, ctypes.byref(p)), "peer_open")
                arenas.append(p.value)
                opened.append(p.value)
            dist.barrier(group=self.group)
        desc = nat.ExchangeDesc(self.size, self.rank, (ctypes.c_void_p * nat.MAX_PEERS)(*arenas), int(nbytes))
        self._arenas[key] = (desc, own.value, opened, device)
        return desc

    def map_peers(self, ptrs: list[int], device: torch.device) -> list[list[int]]:
        """Every rank's address, as mapped in this process, of each device buffer
        in ``ptrs`` (this rank's buffers; every rank calls this collectively with
        its buffers of the same roles): ``out[i][r]`` is rank r's buffer i.  Each
        peer allocation is mapped once (CUDA IPC); ``close`` unmaps them."""
        from . import _native as nat

        key = (tuple(int(p) for p in ptrs), device.index)
        hit = self._peer_maps.get(key)
        if hit is not None:
            return hit
        L = nat.lib()
        mine = []
        with torch.cuda.device(device):
            for p in ptrs:
                h = (ctypes.c_ubyte * nat.IPC_HANDLE_BYTES)()
                off = ctypes.c_int64()
                nat.check(L.kiv_peer_export(ctypes.c_void_p(int(p)), h, ctypes.byref(off)), "peer_export")
                mine.append((bytes(h), int(p) - off.value, off.value))
            everyone = [None] * self.size
            dist.all_gather_object(everyone, mine, group=self.group)
            out = [[0] * self.size for _ in ptrs]
            for r, entries in enumerate(everyone):
                for i, (hb, base, off) in enumerate(entries):
                    if r == self.rank:
                        out[i][r] = int(ptrs[i])
                        continue
                    got = self._peer_bases.get((r, base))
                    if got is None:
                        mp = ctypes.c_void_p()
                        buf = (ctypes.c_ubyte * nat.IPC_HANDLE_BYTES).from_buffer_copy(hb)
                        nat.check(L.kiv_peer_open(buf, ctypes.byref(mp)), "peer_open")
                        got = (mp.value, device)
                        self._peer_bases[(r, base)] = got
                    out[i][r] = got[0] + off
            dist.barrier(group=self.group)
        self._peer_maps[key] = out
        return out

    def close(self) -> None:
        """Unmap the peers' arenas and buffers and free this rank's arenas (after
        all exchanges are done)."""
        from . import _native as nat

        L = nat.lib() if (self._arenas or self._peer_bases) else None
        for desc, own, opened, device in self._arenas.values():
            with torch.cuda.device(device):
                torch.cuda.synchronize(device)
                for p in opened:
                    L.kiv_peer_close(ctypes.c_void_p(p))
        for mapped, device in self._peer_bases.values():
            with torch.cuda.device(device):
                torch.cuda.synchronize(device)
                L.kiv_peer_close(ctypes.c_void_p(mapped))
        had_peers = bool(self._peer_bases)
        self._peer_bases.clear()
        self._peer_maps.clear()
        if self._arenas or had_peers:
            dist.barrier(group=self.group)
        for desc, own, opened, device in self._arenas.values():
            with torch.cuda.device(device):
                L.kiv_peer_free(ctypes.c_void_p(own))
        self._arenas.clear()

    def all_gather(self, out: torch.Tensor, inp: torch.Tensor) -> None:
        """out[n, *inp.shape] <- every rank's ``inp`` (rank order)."""
        dist.all_gather_into_tensor(out.view(-1), inp.contiguous().view(-1), group=self.group)

    def all_reduce_sum(self, t: torch.Tensor) -> None:
        dist.all_reduce(t, op=dist.ReduceOp.SUM, group=self.group)

    def all_or_bits(self, words: torch.Tensor) -> None:
        """Bitwise OR of an int32 bitmap over the ranks, in place (every rank
        ends with the union of all ranks' bits).  The bits travel as bytes
        reduced with MAX, which every backend supports for uint8."""
        shifts = torch.arange(32, device=words.device, dtype=torch.int32)
        flags = ((words[:, None] >> shifts) & 1).to(torch.uint8)
        dist.all_reduce(flags, op=dist.ReduceOp.MAX, group=self.group)
        packed = (flags.to(torch.int64) << shifts.to(torch.int64)).sum(dim=1)
        words.copy_(packed.to(torch.int32))


def shard_of_page(page: int, world: int) -> int:
    """Rank holding global page ``page``."""
    return page % world


def local_page_count(n_pages: int, rank: int, world: int) -> int:
    """Pages of the first ``n_pages`` global pages that live on ``rank``."""
    return (n_pages - rank + world - 1) // world if n_pages > rank else 0
