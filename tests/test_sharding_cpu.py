"""Page-sharded retrieval on CPU ranks (gloo, world size 2).

Every rank holds the same seeded problem, keeps the pages ``p % world ==
rank`` (and, on its owner, the partial page), and runs the sharded layer-step
the GPU path runs: local coarse top-k -> all-gather of (score, page) ->
identical merge -> local fine top-P over its own union pages -> all-gather of
(score, token) -> identical merge -> attention partials over its own selected
tokens and its slice of the hot window -> all-gather -> log-sum-exp merge.
The exchanges go through ``kiv_b200.sharding.ShardComm`` over a real gloo
process group; the per-rank math is the oracle's.  The merged selections must
equal the unsharded oracle's exactly and the merged attention must match it
to 1e-12 (float64).
"""

import os
import socket
import tempfile

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle.kiv_oracle import OracleStore, eager_attention, topk_total_order

WORLD = 2


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _problem(seed=7):
    rng = np.random.default_rng(seed)
    B, Hkv, G, D, S = 1, 2, 3, 32, 16
    n_pages, partial, hot = 41, 5, 24
    ost = OracleStore(B, Hkv, D, G, S, "f32")
    T = n_pages * S + partial
    k = rng.standard_normal((B, Hkv, T, D)).astype(np.float32)
    v = rng.standard_normal((B, Hkv, T, D)).astype(np.float32)
    ost.evict_from_hot(k, v)
    q = rng.standard_normal((B, Hkv * G, 1, D)).astype(np.float32)
    hk = rng.standard_normal((B, Hkv, hot, D))
    hv = rng.standard_normal((B, Hkv, hot, D))
    return ost, q, hk, hv


def _merge_topk(scores: np.ndarray, ids: np.ndarray, k: int) -> np.ndarray:
    """Global top-k of gathered (score, id) lists, ties by lowest id (invalid ids < 0)."""
    ok = ids >= 0
    s, i = scores[ok].astype(np.float64), ids[ok]
    order = np.lexsort((i, -s))
    return np.sort(i[order[:k]])


def _worker(rank, port, out_dir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=WORLD)
    try:
        from kiv_b200.sharding import ShardComm, local_page_count, shard_of_page
        comm = ShardComm()
        assert (comm.rank, comm.size) == (rank, WORLD)

        # the wrapper's collectives on CPU tensors
        t = torch.full((3,), float(rank + 1))
        got = torch.empty(WORLD, 3)
        comm.all_gather(got, t)
        assert got[:, 0].tolist() == [1.0, 2.0]
        comm.all_reduce_sum(t)
        assert t.tolist() == [3.0, 3.0, 3.0]

        ost, q, hk, hv = _problem()
        scaling, top_pages, top_p = 0.25, 6, 50
        Np, S = ost.num_pages, ost.page_size
        owned = np.array([p for p in range(Np) if shard_of_page(p, WORLD) == rank], np.int64)
        assert owned.size == local_page_count(Np, rank, WORLD)

        # ---- coarse: local top-k per row, all-gather, merge
        union_ref, top_ref, sc = ost.coarse(q, scaling, top_pages)
        B, Hq, Q, _ = q.shape
        k = min(top_pages, Np)
        R = B * Hq * Q
        rows = sc.reshape(R, Np)
        ls = np.zeros((R, k), np.float64)
        lp = np.full((R, k), -1, np.int64)
        for r in range(R):
            pos = topk_total_order(rows[r, owned], k)
            ls[r, :pos.size] = rows[r, owned[pos]]
            lp[r, :pos.size] = owned[pos]
        all_s = torch.empty(WORLD, R, k, dtype=torch.float64)
        all_p = torch.empty(WORLD, R, k, dtype=torch.int64)
        comm.all_gather(all_s, torch.from_numpy(ls))
        comm.all_gather(all_p, torch.from_numpy(lp))
        union = set()
        for r in range(R):
            merged = _merge_topk(all_s[:, r].numpy().ravel(), all_p[:, r].numpy().ravel(), k)
            assert merged.tolist() == np.sort(top_ref.reshape(R, -1)[r]).tolist()
            union.update(merged.tolist())
        union = np.array(sorted(union), np.int64)
        assert union.tolist() == union_ref.tolist()

        # ---- fine: own union pages (+ the partial page on its owner), local top-P, merge
        cand_ref = ost.candidates(union)
        agg_ref, sel_ref = ost.fine(q, scaling, cand_ref, top_p)
        mine = np.array([c for c in cand_ref
                         if shard_of_page(int(c) // S, WORLD) == rank], np.int64)
        P = sel_ref.shape[1]
        agg_mine, _ = ost.fine(q, scaling, mine, top_p) if mine.size else (np.zeros((B, 0)), None)
        lt = np.full((B, top_p), -1, np.int64)
        lsc = np.zeros((B, top_p), np.float64)
        for b in range(B):
            pos = topk_total_order(agg_mine[b], min(top_p, mine.size))
            lt[b, :pos.size] = mine[pos]
            lsc[b, :pos.size] = agg_mine[b, pos]
        all_t = torch.empty(WORLD, B, top_p, dtype=torch.int64)
        all_sc = torch.empty(WORLD, B, top_p, dtype=torch.float64)
        comm.all_gather(all_t, torch.from_numpy(lt))
        comm.all_gather(all_sc, torch.from_numpy(lsc))
        for b in range(B):
            merged = _merge_topk(all_sc[:, b].numpy().ravel(), all_t[:, b].numpy().ravel(), P)
            assert merged.tolist() == sel_ref[b].tolist()

        # ---- attention: own selected tokens + own slice of the hot window, LSE merge
        sel_mine = [np.array([t for t in sel_ref[b] if shard_of_page(int(t) // S, WORLD) == rank], np.int64)
                    for b in range(B)]
        hot = hk.shape[2]
        lo, hi = hot * rank // WORLD, hot * (rank + 1) // WORLD
        G = Hq // ost.num_kv_heads
        qq = q.astype(np.float64)
        part = np.zeros((B, Hq, Q, hk.shape[3] + 2))
        for b in range(B):
            kc = ost.k[b][:, sel_mine[b], :].astype(np.float64)
            vc = ost.v[b][:, sel_mine[b], :].astype(np.float64)
            K = np.repeat(np.concatenate([kc, hk[b][:, lo:hi]], axis=1), G, axis=0)
            V = np.repeat(np.concatenate([vc, hv[b][:, lo:hi]], axis=1), G, axis=0)
            s = np.einsum("hqd,hkd->hqk", qq[b], K) * scaling
            m = s.max(axis=-1) if s.shape[-1] else np.full(s.shape[:2], -np.inf)
            p = np.exp(s - m[..., None]) if s.shape[-1] else s
            part[b, ..., :-2] = np.einsum("hqk,hkd->hqd", p, V)
            part[b, ..., -2] = m
            part[b, ..., -1] = p.sum(axis=-1)
        gathered = torch.empty((WORLD,) + part.shape, dtype=torch.float64)
        comm.all_gather(gathered, torch.from_numpy(part))
        g = gathered.numpy()
        M = g[..., -2].max(axis=0)
        w = np.exp(g[..., -2] - M)
        out = (g[..., :-2] * w[..., None]).sum(axis=0) / (g[..., -1] * w).sum(axis=0)[..., None]
        kr, vr = ost.gather(sel_ref)
        ref = eager_attention(q, kr, vr, hk, hv, scaling)                  # [B, Q, Hq, D]
        np.testing.assert_allclose(out.transpose(0, 2, 1, 3), ref, rtol=1e-12, atol=1e-12)
        if rank == 0:
            with open(os.path.join(out_dir, "ok"), "w") as f:
                f.write("ok")
    finally:
        dist.destroy_process_group()


def test_sharded_layer_step_on_gloo_ranks():
    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_worker, args=(_free_port(), d), nprocs=WORLD, join=True, start_method="spawn")
        assert os.path.exists(os.path.join(d, "ok"))


def test_every_shard_allocates_the_same_cold_capacity():
    """Page-sharded stores size their cold slots by the largest shard's page
    count, so every shard's store, workspace and exchange arena share one
    layout (the candidate exchange indexes the arenas by global candidate
    position, and the peer-row attention reads other shards' rows with this
    shard's strides)."""
    from kiv_b200 import ColdKVStore, KIVConfig, ModelTopology

    cfg = KIVConfig(hot_budget=256, page_size=128, top_pages=8, top_p=128)
    topo = ModelTopology.manual(global_layer_indices=(0,), num_query_heads=8, num_kv_heads=1, head_dim=128,
                                num_hidden_layers=1)
    for world in (2, 3, 4, 8):
        stores = [ColdKVStore(cfg, topo, torch.device("cpu"), shard_rank=r, shard_count=world, comm=object())
                  for r in range(world)]
        for tokens in (1, 127, 128, 129, 1000, 4096 + 60, 1 << 20, (1 << 20) + 5):
            caps = {s._round_local(tokens) for s in stores}
            assert len(caps) == 1, (world, tokens, caps)
            cap = caps.pop()
            pages = -(-tokens // 128)
            # enough slots for the pages of the shard holding the most
            assert cap >= max(1, -(-pages // world)) * 128 and cap % 128 == 0


def _cand_worker(rank, port, out_dir, world):
    """The candidate exchange on gloo ranks: every rank holds the whole union
    (replicated summaries), scores the candidates whose page it owns, and
    writes each key at its global candidate position (union position x S +
    token, then the partial page) into a position-indexed array that stands
    for the arenas (here: a sum over the ranks, every position written by
    exactly one); every rank then takes the top-P over all positions, which
    must be the unsharded selection."""
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from kiv_b200.sharding import ShardComm, shard_of_page
        comm = ShardComm()
        ost, q, hk, hv = _problem(seed=11)
        scaling, top_pages, top_p = 0.25, 6, 50
        S = ost.page_size
        union, _, _ = ost.coarse(q, scaling, top_pages)        # the same on every rank
        cand = ost.candidates(union)                             # global candidate positions
        agg_ref, sel_ref = ost.fine(q, scaling, cand, top_p)
        B, C = agg_ref.shape
        owner = np.array([shard_of_page(int(c) // S, world) for c in cand])
        mine = np.nonzero(owner == rank)[0]
        keys = np.zeros((B, C), np.float64)
        wrote = np.zeros(C, np.int64)
        if mine.size:
            agg_mine, _ = ost.fine(q, scaling, cand[mine], top_p)
            keys[:, mine] = agg_mine
            wrote[mine] = 1
        keys_t, wrote_t = torch.from_numpy(keys), torch.from_numpy(wrote)
        comm.all_reduce_sum(keys_t)
        comm.all_reduce_sum(wrote_t)
        assert (wrote_t.numpy() == 1).all(), "every candidate position is written by exactly one rank"
        allk = keys_t.numpy()
        # (the oracle's float32 products over a subset of the candidates may round
        # differently in the last place from the whole set's)
        np.testing.assert_allclose(allk, agg_ref, rtol=1e-6, atol=1e-6)
        P = sel_ref.shape[1]
        for b in range(B):
            got = np.sort(cand[topk_total_order(allk[b], P)])
            assert got.tolist() == sel_ref[b].tolist()
        if rank == 0:
            with open(os.path.join(out_dir, "ok"), "w") as f:
                f.write("ok")
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_candidate_exchange_on_gloo_ranks(world):
    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_cand_worker, args=(_free_port(), d, world), nprocs=world, join=True,
                           start_method="spawn")
        assert os.path.exists(os.path.join(d, "ok"))
