"""CPU tests of the host-side surface: topology invariants and detection,
middleware prefill flow with fake models, mask helpers, synthetic generator,
telemetry key conversion.  Mirrors the reference's tests/test_model_topology.py
and tests/test_middleware.py against kiv_b200."""

from __future__ import annotations

import struct
from types import SimpleNamespace

import pytest
import torch

from kiv_b200.config import KIVConfig
from kiv_b200.hf_topology import detect_topology
from kiv_b200.mask_utils import extend_mask_for_cold
from kiv_b200.middleware import KIVMiddleware, _prefill_logits_kwargs, hot_mask_for_kernel
from kiv_b200.model_topology import ModelTopology
from kiv_b200.synthetic import SynthSpec, make_problem
from kiv_b200.telemetry import _key_to_float


# ------------------------------------------------------------ topology
def _make(**overrides):
    d = dict(model_family="test", num_hidden_layers=4, global_layer_indices=(0, 1, 2),
             independent_kv_layers=(0, 1, 2), kv_sharing_map={}, num_query_heads=2,
             num_kv_heads=1, head_dim=4)
    d.update(overrides)
    return ModelTopology(**d)


def test_valid_topology_constructs():
    t = _make(global_layer_indices=(0, 1, 2, 3), independent_kv_layers=(0, 2), kv_sharing_map={1: 0, 3: 2})
    assert t.kv_sharing_map == {1: 0, 3: 2}


def test_topology_invariants():
    with pytest.raises(ValueError, match="independent_kv_layers"):
        _make(global_layer_indices=(0, 1), independent_kv_layers=(0, 1, 5))
    with pytest.raises(ValueError, match="kv_sharing_map keys"):
        _make(global_layer_indices=(0, 2), independent_kv_layers=(0, 2), kv_sharing_map={1: 0})
    with pytest.raises(ValueError, match="kv_sharing_map values"):
        _make(global_layer_indices=(0, 1, 2), independent_kv_layers=(0,), kv_sharing_map={2: 1})


def test_manual_defaults_to_globals_for_independents():
    t = ModelTopology.manual(global_layer_indices=(0, 1), num_query_heads=2, num_kv_heads=1,
                             head_dim=4, num_hidden_layers=2)
    assert t.independent_kv_layers == (0, 1)


def _fake_model(cfg, shared=None):
    class Attn:
        pass
    layers = []
    for i in range(cfg.num_hidden_layers):
        a = Attn()
        if shared and i in shared:
            a.is_kv_shared_layer = True
            a.kv_shared_layer_index = shared[i]
        layers.append(SimpleNamespace(self_attn=a))
    return SimpleNamespace(config=cfg, model=SimpleNamespace(layers=layers))


def test_detect_topology_layer_types_and_sharing():
    cfg = SimpleNamespace(model_type="gemma3_text", num_hidden_layers=6,
                          layer_types=["sliding_attention", "full_attention"] * 3,
                          num_kv_shared_layers=2, num_attention_heads=8, num_key_value_heads=2,
                          head_dim=64, hidden_size=512)
    t = detect_topology(_fake_model(cfg))
    assert t.global_layer_indices == (1, 3, 5)
    assert t.independent_kv_layers == (1, 3) and t.kv_sharing_map == {5: 3}
    assert (t.num_query_heads, t.num_kv_heads, t.head_dim) == (8, 2, 64)


def test_detect_topology_module_flags_and_geometry_priority():
    cfg = SimpleNamespace(model_type="llama", num_hidden_layers=4, num_attention_heads=8,
                          num_key_value_heads=4, num_global_key_value_heads=1, global_head_dim=256,
                          head_dim=64, hidden_size=512)
    t = detect_topology(_fake_model(cfg, shared={3: 1}))
    assert t.global_layer_indices == (0, 1, 2, 3)
    assert t.kv_sharing_map == {3: 1}
    assert (t.num_kv_heads, t.head_dim) == (1, 256)


# ---------------------------------------------------------- middleware
class _FakeCache:
    def __init__(self):
        self._suppress_cold = False
        self._prefill_complete = False
        self.evict_calls = []
        self.marked = False

    def _evict_to_cap(self, cap):
        self.evict_calls.append(cap)

    def _evict_excess_all_layers(self):
        self.evicted_excess = True

    def mark_prefill_complete(self):
        self.marked = True


class _ModelLTK(torch.nn.Module):
    def __init__(self):
        super().__init__()
        self.config = SimpleNamespace()
        self.calls = []

    def forward(self, input_ids, past_key_values=None, use_cache=False, logits_to_keep=0):
        self.calls.append(logits_to_keep)
        return SimpleNamespace(logits=torch.zeros(input_ids.shape[0], logits_to_keep or input_ids.shape[1], 3))


class _ModelPlain(torch.nn.Module):
    def __init__(self):
        super().__init__()
        self.config = SimpleNamespace()
        self.calls = 0

    def forward(self, input_ids, past_key_values=None, use_cache=False):
        self.calls += 1
        return SimpleNamespace(logits=torch.zeros(input_ids.shape[0], input_ids.shape[1], 3))


def _mw(model):
    mw = KIVMiddleware(model)
    mw._installed = True
    mw._original_impl = "eager"
    mw._kiv_key = "kiv_eager"
    return mw


def test_prefill_logits_kwargs():
    assert _prefill_logits_kwargs(_ModelLTK()) == {"logits_to_keep": 1}
    assert _prefill_logits_kwargs(_ModelPlain()) == {}


def test_chunked_prefill_chunks_and_marks():
    m = _ModelLTK()
    cache = _FakeCache()
    logits = _mw(m).chunked_prefill(torch.ones(1, 5, dtype=torch.long), cache, chunk_size=2)
    assert m.calls == [1, 1, 1] and logits.shape == (1, 3) and cache.marked
    m2 = _ModelPlain()
    logits = _mw(m2).chunked_prefill(torch.ones(1, 5, dtype=torch.long), _FakeCache(), chunk_size=2)
    assert m2.calls == 3 and logits.shape == (1, 3)


def test_chunked_prefill_hot_cap_evicts_each_chunk():
    m = _ModelLTK()
    cache = _FakeCache()
    mw = _mw(m)
    mw.chunked_prefill(torch.ones(1, 7, dtype=torch.long), cache, chunk_size=3, prefill_hot_cap=4)
    assert cache.evict_calls == [4, 4, 4]
    assert cache._prefill_complete is True and not cache.marked
    assert cache._suppress_cold is False
    assert m.config._attn_implementation == "kiv_eager"


def test_chunked_prefill_empty_cache_opt_in(monkeypatch):
    calls = []
    monkeypatch.setattr(torch.cuda, "empty_cache", lambda: calls.append(True))
    _mw(_ModelLTK()).chunked_prefill(torch.ones(1, 10, dtype=torch.long), _FakeCache(), chunk_size=1)
    assert calls == []
    _mw(_ModelLTK()).chunked_prefill(torch.ones(1, 5, dtype=torch.long), _FakeCache(), chunk_size=1,
                                      empty_cache_interval=2)
    assert calls == [True, True]


def test_chunked_prefill_restores_impl_on_error():
    class Boom(_ModelLTK):
        def forward(self, *a, **k):
            raise RuntimeError("boom")
    m = Boom()
    cache = _FakeCache()
    with pytest.raises(RuntimeError):
        _mw(m).chunked_prefill(torch.ones(1, 4, dtype=torch.long), cache, chunk_size=2, prefill_hot_cap=2)
    assert m.config._attn_implementation == "kiv_eager" and cache._suppress_cold is False


def test_create_cache_requires_install():
    with pytest.raises(RuntimeError):
        KIVMiddleware(_ModelPlain()).create_cache()


# --------------------------------------------------------------- masks
def test_extend_mask_for_cold():
    m = torch.zeros(2, 1, 3, 5)
    e = extend_mask_for_cold(m, 4)
    assert e.shape == (2, 1, 3, 9) and torch.all(e[..., :4] == 0)
    b = extend_mask_for_cold(torch.zeros(2, 5, dtype=torch.bool), 3)
    assert b.shape == (2, 8) and b[:, :3].all()


def test_hot_mask_for_kernel():
    m, causal = hot_mask_for_kernel(None, 10, 1)
    assert m is None and causal is False
    m, causal = hot_mask_for_kernel(None, 10, 4)
    assert m is None and causal is True
    full = torch.zeros(1, 1, 2, 12)
    full[..., -1] = float("-inf")
    m, causal = hot_mask_for_kernel(full, 10, 2)
    assert m.shape == (1, 1, 2, 10) and m.dtype == torch.float32 and torch.isinf(m[..., -1]).all()
    bm = torch.ones(1, 1, 1, 10, dtype=torch.bool)
    bm[..., 0] = False
    m, _ = hot_mask_for_kernel(bm, 10, 1)
    assert m[0, 0, 0, 0] == float("-inf") and m[0, 0, 0, 1] == 0
    pm = torch.tensor([[0, 1, 1, 1]])
    m, causal = hot_mask_for_kernel(pm, 4, 2)
    assert m.shape == (1, 1, 2, 4) and causal is True and m[0, 0, 0, 0] == float("-inf")


# ----------------------------------------------------------- synthetic
def test_synthetic_is_deterministic_and_plants_needle():
    spec = SynthSpec(batch=1, num_query_heads=4, num_kv_heads=2, head_dim=16, cold_tokens=1024,
                     hot_budget=64, page_size=128)
    a = make_problem(spec, seed=3)
    b = make_problem(spec, seed=3)
    assert torch.equal(a.prefill_k, b.prefill_k) and torch.equal(a.query, b.query)
    p = a.needle_page
    assert 0 <= p < 8
    q = a.query.float().mean(dim=2).view(1, 2, 2, 16).mean(dim=2)
    qhat = q / q.norm(dim=-1, keepdim=True)
    page = a.prefill_k[:, :, p * 128:(p + 1) * 128].mean(dim=2)
    assert torch.allclose(page, 2 * qhat, atol=0.1)


def test_key_to_float_roundtrip():
    for f in (0.0, 1.5, -2.25, 1e-3, -7e4):
        u = struct.unpack("<I", struct.pack("<f", f))[0]
        key = (~u & 0xFFFFFFFF) if (u & 0x80000000) else (u | 0x80000000)
        assert abs(_key_to_float(key) - f) <= abs(f) * 1e-7


def test_config_defaults_match_reference():
    c = KIVConfig()
    assert (c.hot_budget, c.top_p, c.page_size, c.top_pages, c.prefetch_stream) == (2048, 256, 128, 32, True)


class _Store(SimpleNamespace):
    pass


class _ReuseCache(_FakeCache):
    def __init__(self):
        super().__init__()
        self._prefill_complete = True
        self.cold_stores = {0: _Store(_cached_candidate_k=1, _cached_candidate_v=1, _cached_candidate_idx=1,
                                      _cached_step=5)}
        self.flags_seen, self.excess = [], 0

    def _evict_excess_all_layers(self):
        self.excess += 1


class _ModelSeesFlag(_ModelPlain):
    def __init__(self, cache):
        super().__init__()
        self.cache = cache

    def forward(self, input_ids, past_key_values=None, use_cache=False):
        st = self.cache.cold_stores[0]
        self.cache.flags_seen.append((self.cache._prefill_complete, st._cached_step, st._cached_candidate_idx))
        st._cached_step = 9              # a retrieval inside the chunk sets the reuse key again
        return super().forward(input_ids, past_key_values, use_cache)


def test_chunked_reuse_prefill_semantics():
    from kiv_b200.middleware import chunked_reuse_prefill
    cache = _ReuseCache()
    m = _ModelSeesFlag(cache)
    logits = chunked_reuse_prefill(m, torch.ones(1, 7, dtype=torch.long), cache, chunk_size=3)
    assert m.calls == 3 and logits.shape == (1, 3)
    # every chunk ran without eviction and with the candidate reuse dropped
    assert cache.flags_seen == [(False, -1, None)] * 3
    assert cache.excess == 3 and cache._prefill_complete is True


def test_chunked_reuse_prefill_restores_flag_on_error():
    from kiv_b200.middleware import chunked_reuse_prefill

    class Boom(_ModelPlain):
        def forward(self, *a, **k):
            raise RuntimeError("boom")
    cache = _ReuseCache()
    cache._prefill_complete = False
    with pytest.raises(RuntimeError):
        chunked_reuse_prefill(Boom(), torch.ones(1, 4, dtype=torch.long), cache, chunk_size=2)
    assert cache._prefill_complete is False
