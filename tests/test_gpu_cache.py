"""GPU tests of the cache contracts the reference pins in ``tests/test_cache.py``,
plus eviction, growth and hot-window bookkeeping of the HBM tiers."""

import numpy as np
import pytest
import torch
from transformers import PretrainedConfig

from kiv_b200 import ColdKVStore, KIVConfig, ModelTopology, TieredKVCache
from kiv_b200 import _native as nat
from oracle.kiv_oracle import OracleStore, page_summary
from tests.gpu_helpers import DEV

pytestmark = pytest.mark.gpu


def _topology(*, global_layer_indices=(0,), independent_kv_layers=(0,), kv_sharing_map=None,
              num_hidden_layers=1, hq=2, hkv=1, d=4):
    return ModelTopology.manual(global_layer_indices=global_layer_indices,
                                independent_kv_layers=independent_kv_layers,
                                kv_sharing_map=kv_sharing_map or {}, num_query_heads=hq,
                                num_kv_heads=hkv, head_dim=d, num_hidden_layers=num_hidden_layers)


def test_retrieve_top_kv_preserves_batch_dimension():
    # reference tests/test_cache.py:30-44
    config = KIVConfig(page_size=2, top_p=1, top_pages=1, prefetch_stream=False)
    store = ColdKVStore(config, _topology(), DEV)
    key = torch.randn(2, 1, 2, 4, device=DEV)
    value = torch.randn(2, 1, 2, 4, device=DEV)
    query = torch.randn(2, 2, 1, 4, device=DEV)
    store.evict_from_hot(key, value)
    ck, cv = store.retrieve_top_kv(query, 1.0, config)
    assert ck.shape == (2, 1, 1, 4) and cv.shape == (2, 1, 1, 4)
    assert torch.cat([ck, torch.randn(2, 1, 1, 4, device=DEV)], dim=2).shape == (2, 1, 2, 4)


def test_empty_store_returns_none():
    config = KIVConfig(page_size=4)
    store = ColdKVStore(config, _topology(), DEV)
    assert store.retrieve_top_kv(torch.randn(1, 2, 1, 4, device=DEV), 1.0, config) == (None, None)


def test_shared_layer_seq_length_resolves_to_source_layer():
    topo = _topology(global_layer_indices=(0, 1), independent_kv_layers=(0,), kv_sharing_map={1: 0},
                     num_hidden_layers=2)
    cache = TieredKVCache(PretrainedConfig(num_hidden_layers=2), KIVConfig(prefetch_stream=False), topo, DEV)
    cache._total_tokens[0] = 123
    assert cache.get_seq_length(0) == 123 and cache.get_seq_length(1) == 123
    assert cache.get_cold_store(1) is cache.get_cold_store(0)


def _cache(hot_budget=2048, page_size=128):
    return TieredKVCache(PretrainedConfig(num_hidden_layers=1),
                         KIVConfig(hot_budget=hot_budget, page_size=page_size, prefetch_stream=False),
                         _topology(), DEV)


def test_truncate_to_hot_only_succeeds():
    cache = _cache()
    key = torch.randn(1, 1, 10, 4, device=DEV)
    value = torch.randn(1, 1, 10, 4, device=DEV)
    cache.update(key, value, 0)
    assert cache.truncate_to(6) is True
    layer = cache.layers[0]
    assert layer.keys.shape[2] == 6 and layer.values.shape[2] == 6
    assert cache._total_tokens[0] == 6
    torch.testing.assert_close(layer.keys, key[:, :, :6, :])
    torch.testing.assert_close(layer.values, value[:, :, :6, :])


def test_truncate_to_rejects_lengths_beyond_current_total():
    cache = _cache()
    cache.update(torch.randn(1, 1, 4, 4, device=DEV), torch.randn(1, 1, 4, 4, device=DEV), 0)
    assert cache.truncate_to(10) is False
    assert cache.layers[0].keys.shape[2] == 4


def test_truncate_to_rejects_truncation_into_cold():
    cache = _cache(hot_budget=4, page_size=2)
    cache.update(torch.randn(1, 1, 10, 4, device=DEV), torch.randn(1, 1, 10, 4, device=DEV), 0)
    cache.mark_prefill_complete()
    assert cache.cold_stores[0].cold_length == 6
    assert cache.truncate_to(3) is False
    assert cache.truncate_to(6) is True
    assert cache.layers[0].keys.shape[2] == 0


def test_device_state_tracks_host_mirror_through_many_steps():
    """Decode 700 steps with a small hot budget: hot compactions, cold growth and
    page finalization all happen; the device state must equal the host mirror
    and the cold rows / summaries must equal the oracle's."""
    S, budget = 16, 40
    cfg = KIVConfig(hot_budget=budget, page_size=S, hot_slack=8, cold_capacity=64)
    topo = _topology(hq=4, hkv=2, d=8)
    cache = TieredKVCache(PretrainedConfig(num_hidden_layers=1), cfg, topo, DEV)
    g = torch.Generator().manual_seed(3)
    pk, pv = torch.randn(1, 2, 100, 8, generator=g), torch.randn(1, 2, 100, 8, generator=g)
    cache.update(pk.to(DEV), pv.to(DEV), 0)
    cache.mark_prefill_complete()
    ost = OracleStore(1, 2, 8, 2, S, "f32")
    ost.evict_from_hot(pk[:, :, :60].numpy(), pv[:, :, :60].numpy())
    hot_k = [pk[:, :, 60:]]
    for _ in range(700):
        k, v = torch.randn(1, 2, 1, 8, generator=g), torch.randn(1, 2, 1, 8, generator=g)
        cache.update(k.to(DEV), v.to(DEV), 0)
        allk = torch.cat(hot_k + [k], dim=2)
        ost.evict_from_hot(allk[:, :, :1].numpy(), allk[:, :, :1].numpy() * 0)
        hot_k = [allk[:, :, 1:]]
    store = cache.get_cold_store(0)
    st = store.read_state()
    assert st[nat.ST_COLD_LEN] == store.cold_length == 760
    assert st[nat.ST_HOT_LEN] == store.hot_length == budget
    assert st[nat.ST_HOT_START] == store._hot_start
    assert st[nat.ST_ERROR] == 0
    torch.testing.assert_close(cache.layers[0].keys.cpu(), hot_k[0], rtol=0, atol=0)
    cold_k = store._k[:, :, :store.cold_length].cpu().numpy()
    np.testing.assert_array_equal(cold_k, ost.k)
    np.testing.assert_array_equal(store.page_summaries().cpu().numpy(), ost.summaries)


def test_evict_to_cap_then_budget_matches_one_shot_prefill():
    """Bounded prefill (evict to a cap after each chunk) ends in the same cold
    state as prefill-then-evict (kiv/middleware.py:238-258)."""
    S = 8
    g = torch.Generator().manual_seed(5)
    k, v = torch.randn(1, 2, 300, 16, generator=g), torch.randn(1, 2, 300, 16, generator=g)
    topo = _topology(hq=4, hkv=2, d=16)
    a = TieredKVCache(PretrainedConfig(num_hidden_layers=1), KIVConfig(hot_budget=32, page_size=S), topo, DEV)
    a.update(k.to(DEV), v.to(DEV), 0)
    a.mark_prefill_complete()
    b = TieredKVCache(PretrainedConfig(num_hidden_layers=1), KIVConfig(hot_budget=32, page_size=S), topo, DEV)
    for c in range(0, 300, 64):
        b.update(k[:, :, c:c + 64].to(DEV), v[:, :, c:c + 64].to(DEV), 0)
        b._evict_to_cap(50)
    b._prefill_complete = True
    b._evict_excess_all_layers()
    sa, sb = a.get_cold_store(0), b.get_cold_store(0)
    assert sa.cold_length == sb.cold_length == 268
    assert torch.equal(sa._k[:, :, :268], sb._k[:, :, :268])
    assert torch.equal(sa.page_summaries(), sb.page_summaries())
    assert torch.equal(a.layers[0].keys, b.layers[0].keys)


def test_bad_shapes_raise_not_fault():
    """Host-side validation turns bad arguments into exceptions before launch."""
    cfg = KIVConfig(page_size=8)
    store = ColdKVStore(cfg, _topology(hq=4, hkv=2, d=6), DEV)   # 6 fp32 = 24 B rows
    with pytest.raises(nat.KIVNativeError):
        store.evict_from_hot(torch.randn(1, 2, 8, 6, device=DEV), torch.randn(1, 2, 8, 6, device=DEV))


def test_memory_report_keys():
    cache = _cache(hot_budget=16, page_size=8)
    cache.update(torch.randn(1, 1, 40, 4, device=DEV), torch.randn(1, 1, 40, 4, device=DEV), 0)
    cache.mark_prefill_complete()
    rep = cache.memory_report()
    for key in ("hot_vram_bytes", "k_index_cpu_bytes", "v_store_cpu_bytes", "page_summaries_gpu_bytes",
                "total_vram_bytes", "total_cpu_bytes"):
        assert key in rep
    assert rep["hot_vram_bytes"] == 2 * 16 * 4 * 4
    assert rep["page_summaries_gpu_bytes"] == 3 * 4 * 4


def test_telemetry_snapshot_format():
    cfg = KIVConfig(hot_budget=8, page_size=4, top_pages=2, top_p=3)
    cache = TieredKVCache(PretrainedConfig(num_hidden_layers=1), cfg, _topology(hq=2, hkv=1, d=4), DEV)
    cache.update(torch.randn(1, 1, 30, 4, device=DEV), torch.randn(1, 1, 30, 4, device=DEV), 0)
    cache.mark_prefill_complete()
    store = cache.get_cold_store(0)
    q = torch.randn(1, 2, 1, 4, device=DEV)
    store.retrieve_top_kv(q, 0.5, cfg, step=1)
    store.retrieve_top_kv(q, 0.5, cfg, step=1)   # reuse -> coarse skipped
    snap = store.telemetry_snapshot()
    agg = snap["aggregates"]
    assert agg["coarse_calls"] == agg["fine_calls"] == 2
    assert agg["coarse_real_calls"] == 1 and agg["coarse_skipped_calls"] == 1
    coarse = [r for r in snap["recent"] if r["kind"] == "coarse"]
    fine = [r for r in snap["recent"] if r["kind"] == "fine"]
    assert coarse[0]["num_pages"] == 5 and 2 <= coarse[0]["num_pages_selected"] <= 4
    assert coarse[1]["skipped"] is True
    assert len(fine[0]["selected_token_indices"]) == 3
    # top / mean scores agree with a direct computation
    summ = store.page_summaries()[0, 0].float()
    sc = (q[0, :, 0].float() @ summ.T) * 0.5
    assert abs(coarse[0]["top_score"] - sc.max().item()) < 1e-5
    assert abs(coarse[0]["mean_score"] - sc.mean().item()) < 1e-5
