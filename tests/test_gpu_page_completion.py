"""Decode steps that finalize a page, on the tensor-core (tcgen05) scoring path.

The eviction kernel of a decode step writes the summary of a page that the
step completes, and the coarse scorer launched right after it (programmatic
dependent launch) must score that page from the new summary.  Here the page
that completes during the steps is a strong match for the query, so a stale
or half-written summary of it would drop it from the coarse union: at every
step the union and the token set must equal the oracle's (ties within 1e-6),
and the completed page must be selected once it is final.  Both the eager
steps and the captured decode graph are checked.
"""

import numpy as np
import pytest
import torch
from transformers import PretrainedConfig

from kiv_b200 import KIVConfig, ModelTopology, TieredKVCache
from kiv_b200.decode_graph import DecodeGraph
from oracle.kiv_oracle import OracleLayer, OracleStore, eager_attention
from tests.gpu_helpers import DEV, check_selection, kernel_union, rel_err

pytestmark = pytest.mark.gpu

S, D, HQ, HKV = 128, 128, 8, 2
PAGES = 40            # finalized pages after the prefill
PART = 120            # rows of the partial page after the prefill
HOT = 256


def _data(seed):
    g = torch.Generator().manual_seed(seed)
    n = PAGES * S + PART + HOT
    cent = torch.randn(1, HKV, n // 512 + 2, D, generator=g) / 8.0
    seg = torch.arange(n) // 512
    k = cent[:, :, seg] + 0.3 * torch.randn(1, HKV, n, D, generator=g)
    v = torch.randn(1, HKV, n, D, generator=g)
    q = torch.randn(1, HQ, 1, D, generator=g)
    qhat = q.reshape(1, HKV, HQ // HKV, D).mean(2)
    qhat = qhat / qhat.norm(dim=-1, keepdim=True)
    # the rows that complete page PAGES (the partial page's rows and the first
    # decode steps' evictions, which come from the prefill's hot tail) match q
    k[:, :, PAGES * S:(PAGES + 1) * S] = 2.0 * qhat[:, :, None] + 0.3 * torch.randn(1, HKV, S, D, generator=g)
    steps_k = 2.0 * qhat[:, :, None] + 0.3 * torch.randn(1, HKV, 24, D, generator=g)
    steps_v = torch.randn(1, HKV, 24, D, generator=g)
    bf = lambda t: t.to(torch.bfloat16)
    return bf(k), bf(v), bf(q), bf(steps_k), bf(steps_v)


def _cache():
    cfg = KIVConfig(hot_budget=HOT, page_size=S, top_pages=4, top_p=256, telemetry=False,
                    cold_capacity=(PAGES + 4) * S)
    topo = ModelTopology.manual(global_layer_indices=(0,), num_query_heads=HQ, num_kv_heads=HKV,
                                head_dim=D, num_hidden_layers=1)
    return cfg, TieredKVCache(PretrainedConfig(num_hidden_layers=1), cfg, topo, DEV)


def _oracle(k, v):
    ol = OracleLayer(OracleStore(1, HKV, D, HQ // HKV, S, "bf16"), HOT)
    ol.update(k.float().numpy(), v.float().numpy())
    ol.mark_prefill_complete()
    return ol


def test_page_completed_during_decode_is_scored_fresh():
    k, v, q, sk, sv = _data(5)
    cfg, cache = _cache()
    cache.update(k.to(DEV), v.to(DEV), 0)
    cache.mark_prefill_complete()
    store = cache.get_cold_store(0)
    ol = _oracle(k, v)
    assert store.cold_length == PAGES * S + PART
    scaling = D ** -0.5
    qd = q.to(DEV)
    completed = False
    for i in range(sk.shape[2]):
        cache.update(sk[:, :, i:i + 1].to(DEV), sv[:, :, i:i + 1].to(DEV), 0)
        ol.update(sk[:, :, i:i + 1].float().numpy(), sv[:, :, i:i + 1].float().numpy())
        out = store.attend(qd, scaling, cfg, step=cache._decode_step)
        sel, P = store.retrieve_indices(qd, scaling, cfg)
        check_selection(store, ol, q.float().numpy(), scaling, cfg, sel, P, storage="bf16")
        assert store.read_state()[7] == 0, "kernel error bits"
        if store.cold_length >= (PAGES + 1) * S:
            completed = True
            assert PAGES in set(kernel_union(store, 1, HQ, 1, cfg).tolist()), \
                f"step {i}: the completed page is missing from the union"
        ko, vo = ol.store.gather(sel[:, :P].cpu().numpy())
        ref = eager_attention(q.float().numpy(), ko, vo, ol.hot_k, ol.hot_v, scaling)
        assert rel_err(out.float().cpu().numpy(), ref) <= 2e-2, f"step {i}"
    assert completed


def test_page_completion_inside_decode_graph_matches_eager():
    """The same steps replayed from a captured decode graph give the eager outputs."""
    k, v, q, sk, sv = _data(6)
    scaling = D ** -0.5
    outs = []
    for mode in ("eager", "graph"):
        cfg, cache = _cache()
        cache.update(k.to(DEV), v.to(DEV), 0)
        cache.mark_prefill_complete()
        store = cache.get_cold_store(0)
        res = []
        if mode == "eager":
            for i in range(sk.shape[2]):
                cache.update(sk[:, :, i:i + 1].to(DEV), sv[:, :, i:i + 1].to(DEV), 0)
                res.append(store.attend(q.to(DEV), scaling, cfg, step=cache._decode_step).float().cpu())
        else:
            sq = q.to(DEV)[None].clone()
            skk = torch.empty(1, 1, HKV, 1, D, dtype=torch.bfloat16, device=DEV)
            svv = torch.empty_like(skk)
            out = torch.empty(1, 1, 1, HQ, D, dtype=torch.bfloat16, device=DEV)
            graph = None
            for i in range(sk.shape[2]):
                skk.copy_(sk[:, :, i:i + 1].to(DEV)[None])
                svv.copy_(sv[:, :, i:i + 1].to(DEV)[None])
                if graph is None:
                    # capture runs the first step for real (warm-up), then records it
                    graph = DecodeGraph(cache, [0], scaling, sq, skk, svv, out, max_steps=64)
                else:
                    graph.replay()
                res.append(out[0].float().cpu().clone())
        assert store.read_state()[7] == 0
        assert store.cold_length >= (PAGES + 1) * S
        outs.append(res)
    for i, (a, b) in enumerate(zip(*outs)):
        assert torch.equal(a, b), f"step {i}: graph replay differs from the eager step"
