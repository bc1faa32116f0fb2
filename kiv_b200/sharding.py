"""Collectives of the page-sharded cold tier (one process per GPU, NCCL over NVLink).

The cold tier of a layer is partitioned by page over the GPUs of one box (page
p lives on rank p % world).  A decode layer-step then needs three small
exchanges, all all-gathers of a few KB to tens of KB (latency-bound):
per-row coarse candidates (score, page), per-batch-row fine candidates
(score, token) and per-row attention partials (out, max, sum).  Each rank
merges the gathered lists identically, so every rank ends with the exact
global top-k and the same merged output.
"""

from __future__ import annotations

import torch
import torch.distributed as dist


class ShardComm:
    """Thin wrapper over a ``torch.distributed`` process group."""

    def __init__(self, group=None) -> None:
        self.group = group
        self.rank = dist.get_rank(group)
        self.size = dist.get_world_size(group)

    def all_gather(self, out: torch.Tensor, inp: torch.Tensor) -> None:
        """out[n, *inp.shape] <- every rank's ``inp`` (rank order)."""
        dist.all_gather_into_tensor(out.view(-1), inp.contiguous().view(-1), group=self.group)

    def all_reduce_sum(self, t: torch.Tensor) -> None:
        dist.all_reduce(t, op=dist.ReduceOp.SUM, group=self.group)


def shard_of_page(page: int, world: int) -> int:
    """Rank holding global page ``page``."""
    return page % world


def local_page_count(n_pages: int, rank: int, world: int) -> int:
    """Pages of the first ``n_pages`` global pages that live on ``rank``."""
    return (n_pages - rank + world - 1) // world if n_pages > rank else 0
