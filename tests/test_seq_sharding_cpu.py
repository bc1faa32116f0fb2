"""Sequence-sharded retrieval on CPU ranks (gloo, world size 2).

A batch of four sequences is split over two ranks (two each).  The reference
takes the page union across the whole batch (kiv/cold_store.py:224), so every
sequence sees pages chosen by any other; sharded, each rank marks the pages
its own sequences' rows choose, the ranks OR the page bitmaps
(``ShardComm.all_or_bits``, the exchange ``ColdKVStore`` runs between the
coarse and fine passes with a ``batch_group``), and each rank's fine pass over
the merged union must select exactly what the unsharded oracle selects for
those sequences.  The bitmap OR itself is checked on words with the sign bit
set.
"""

import os
import socket
import tempfile

import numpy as np
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle.kiv_oracle import OracleStore

WORLD = 2


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _store(k, v, G, S):
    B, H, _, D = k.shape
    st = OracleStore(B, H, D, G, S, "f32")
    st.evict_from_hot(k, v)
    return st


def _worker(rank, port, out_dir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=WORLD)
    try:
        from kiv_b200.sharding import ShardComm
        comm = ShardComm()

        # OR of bitmaps, including the sign bit of an int32 word
        mine = torch.tensor([1 << rank, -2 ** 31 if rank == 0 else 0, 0x0F0 if rank else 0x00F], dtype=torch.int32)
        comm.all_or_bits(mine)
        assert mine.tolist() == [3, -2 ** 31, 0x0FF]

        rng = np.random.default_rng(5)
        B, H, G, D, S = 4, 2, 3, 16, 8
        n_pages, partial = 37, 3
        T = n_pages * S + partial
        k = rng.standard_normal((B, H, T, D)).astype(np.float32)
        v = rng.standard_normal((B, H, T, D)).astype(np.float32)
        q = rng.standard_normal((B, H * G, 1, D)).astype(np.float32)
        scaling, top_pages, top_p = 0.25, 3, 20
        full = _store(k, v, G, S)
        union_ref, _, _ = full.coarse(q, scaling, top_pages)
        agg_ref, sel_ref = full.fine(q, scaling, full.candidates(union_ref), top_p)

        lo, hi = 2 * rank, 2 * rank + 2
        local = _store(k[lo:hi], v[lo:hi], G, S)
        union_mine, _, _ = local.coarse(q[lo:hi], scaling, top_pages)
        words = torch.zeros((n_pages + 31) // 32, dtype=torch.int32)
        for p in union_mine.tolist():
            w, b = divmod(int(p), 32)
            words[w] = int(np.int32(np.uint32(int(words[w]) & 0xFFFFFFFF | (1 << b))))
        comm.all_or_bits(words)
        bits = [(int(words[p // 32]) >> (p % 32)) & 1 for p in range(n_pages)]
        union = np.array([p for p in range(n_pages) if bits[p]], np.int64)
        assert union.tolist() == union_ref.tolist(), (union, union_ref)
        assert set(union_mine.tolist()) < set(union.tolist()) or set(union_mine.tolist()) == set(union.tolist())
        _, sel = local.fine(q[lo:hi], scaling, local.candidates(union), top_p)
        assert np.array_equal(sel, sel_ref[lo:hi])
        if rank == 0:
            with open(os.path.join(out_dir, "ok"), "w") as f:
                f.write("ok")
    finally:
        dist.destroy_process_group()


def test_sequence_sharded_union_on_gloo_ranks():
    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_worker, args=(_free_port(), d), nprocs=WORLD, join=True, start_method="spawn")
        assert os.path.exists(os.path.join(d, "ok"))
