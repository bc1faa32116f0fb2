"""Exchanges of the sharded cold tier (one process per GPU of one box).

Two partitions exist.  Sequence sharding (``batch_group``): each rank holds
its own sequences of the batch; the only exchange is the page union, which
the reference takes across the whole batch (kiv/cold_store.py:224) -- the
ranks OR their coarse page marks (``all_or_bits``) before the fine pass, and
everything after it is per sequence.  Page sharding (``shard_group``) splits
one sequence's cold pages:

The cold tier of a layer is partitioned by page over the GPUs of one box (page
p lives on rank p % world).  A decode layer-step then needs three small
exchanges of a few KB to tens of KB (latency-bound): per-row coarse
candidates (score, page), per-batch-row fine candidates (score, token) and
per-row attention partials (out, max, sum).  Each rank merges the gathered
lists identically, so every rank ends with the exact global top-k and the same
merged output.

On CUDA the exchanges go through peer memory: every rank allocates an
exchange arena, the ranks swap CUDA IPC handles once over the process group,
and the merge kernels store their lists straight into the peers' arenas over
NVLink as words that carry the exchange's flag, and wait (bounded) until every
rank's words carry it (``kiv_*_exchange_merge`` in the C ABI).  ``all_gather`` / ``all_reduce_sum`` (the process group's collectives)
remain for the API paths that return tensors and for CPU process groups.
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

    def close(self) -> None:
        """Unmap the peers' arenas and free this rank's (after all exchanges are done)."""
        from . import _native as nat

        L = nat.lib() if self._arenas else None
        for desc, own, opened, device in self._arenas.values():
            with torch.cuda.device(device):
                torch.cuda.synchronize(device)
                for p in opened:
                    L.kiv_peer_close(ctypes.c_void_p(p))
        if self._arenas:
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
