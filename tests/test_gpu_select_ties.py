"""Exact ties in both selections, on the 16-bit tensor-core decode path.

Every cold key is the same vector, so every page summary, every coarse score
and every fine score of a row is equal.  The reference's order breaks ties by
the lowest index (the oracle's total order: score descending, index
ascending), so the coarse union must be exactly the first `top_pages` pages
and the selected tokens exactly the first `top_p` tokens.  600 pages: the
threshold-bin pages are ranked directly; 1100 pages: more tied pages than the
coarse top-k's boundary buffer, so its general path resolves them.
"""

import pytest
import torch
from transformers import PretrainedConfig

from kiv_b200 import KIVConfig, ModelTopology, TieredKVCache
from tests.gpu_helpers import DEV, kernel_union

pytestmark = pytest.mark.gpu

S, D, HQ, HKV, HOT = 128, 128, 8, 1, 256


@pytest.mark.parametrize("pages", [600, 1100])
def test_all_equal_scores_select_lowest_indices(pages):
    cfg = KIVConfig(hot_budget=HOT, page_size=S, top_pages=8, top_p=256, telemetry=False)
    topo = ModelTopology.manual(global_layer_indices=(0,), num_query_heads=HQ, num_kv_heads=HKV,
                                head_dim=D, num_hidden_layers=1)
    cache = TieredKVCache(PretrainedConfig(num_hidden_layers=1), cfg, topo, DEV)
    g = torch.Generator().manual_seed(4)
    n = pages * S + HOT
    c = torch.randn(D, generator=g) * 0.2
    k = c.expand(1, HKV, n, D).to(torch.bfloat16).contiguous()
    v = torch.randn(1, HKV, n, D, generator=g).to(torch.bfloat16)
    cache.update(k.to(DEV), v.to(DEV), 0)
    cache.mark_prefill_complete()
    step_k = c.expand(1, HKV, 1, D).to(torch.bfloat16).contiguous()
    cache.update(step_k.to(DEV), torch.randn(1, HKV, 1, D, generator=g).to(torch.bfloat16).to(DEV), 0)
    store = cache.get_cold_store(0)
    assert store.cold_length == pages * S + 1
    q = torch.randn(1, HQ, 1, D, generator=g).to(torch.bfloat16).to(DEV)
    sel, P = store.retrieve_indices(q, D ** -0.5, cfg)
    assert store.read_state()[7] == 0, "kernel error bits"
    assert kernel_union(store, 1, HQ, 1, cfg).tolist() == list(range(cfg.top_pages))
    assert P == cfg.top_p
    assert sel[0, :P].tolist() == list(range(cfg.top_p))
