"""vLLM integration host logic on CPU: topology from a vLLM config, the
connector's layer routing / row extraction / step tracking, and the attention
hook's reshapes, module discovery and install/uninstall
(tests/test_vllm_topology.py, tests/test_vllm_connector.py,
tests/test_vllm_attention_hook.py of the reference).  Stores are recording
fakes where a test would otherwise launch kernels."""

from types import SimpleNamespace
from unittest.mock import MagicMock

import pytest
import torch

from kiv_b200 import ModelTopology
from kiv_b200.vllm import attention_hook as hook
from kiv_b200.vllm.connector import KIVConnector, _new_rows, _parse_layer_index
from kiv_b200.vllm.topology import (_detect_global_layers, _detect_head_geometry, _detect_kv_sharing,
                                    detect_topology_from_vllm)


def _hf(**kw):
    d = dict(num_hidden_layers=26, num_attention_heads=8, num_key_value_heads=1, head_dim=256,
             hidden_size=2048)
    d.update(kw)
    return SimpleNamespace(**d)


def _vllm_config(hf=None, **kiv):
    hf = hf or SimpleNamespace(model_type="llama", num_hidden_layers=4, num_attention_heads=8,
                               num_key_value_heads=2, head_dim=64, hidden_size=512)
    return SimpleNamespace(model_config=SimpleNamespace(hf_config=hf), extra_config={"kiv": kiv} if kiv else {})


def _topo(glob, indep, sharing=None):
    return ModelTopology(model_family="test", num_hidden_layers=4, global_layer_indices=glob,
                         independent_kv_layers=indep, kv_sharing_map=sharing or {}, num_query_heads=8,
                         num_kv_heads=2, head_dim=64)


class RecordingStore:
    """Stand-in for ColdKVStore: records the rows handed to evict_from_hot."""

    def __init__(self):
        self.calls = []

    def evict_from_hot(self, k, v):
        self.calls.append((k.clone(), v.clone()))

    @property
    def cold_length(self):
        return sum(k.shape[2] for k, _ in self.calls)


# ---------------------------------------------------------------- topology

def test_global_layers_from_layer_types():
    assert _detect_global_layers(_hf(layer_types=["sliding_attention", "full_attention"] * 13)) == \
        tuple(range(1, 26, 2))


def test_global_layers_all_when_no_full_attention_named():
    assert _detect_global_layers(_hf(layer_types=["sliding_attention"] * 26)) == tuple(range(26))


@pytest.mark.parametrize("extra", [{}, {"sliding_window": 4096}])
def test_global_layers_default_all(extra):
    assert _detect_global_layers(_hf(**extra)) == tuple(range(26))


def test_kv_sharing_none():
    g = tuple(range(26))
    assert _detect_kv_sharing(_hf(), g) == (g, {})


def test_kv_sharing_from_num_kv_shared_layers():
    indep, sharing = _detect_kv_sharing(_hf(num_kv_shared_layers=12), (0, 6, 12, 18, 24))
    assert indep == (0, 6, 12)
    assert sharing == {18: 12, 24: 12}


def test_kv_sharing_all_shared_keeps_globals_independent():
    assert _detect_kv_sharing(_hf(num_kv_shared_layers=26), (3, 5)) == ((3, 5), {})


def test_head_geometry_variants():
    assert _detect_head_geometry(_hf(num_key_value_heads=2, head_dim=128)) == (8, 2, 128)
    mha = _hf(num_attention_heads=32, hidden_size=4096)
    del mha.num_key_value_heads, mha.head_dim
    assert _detect_head_geometry(mha) == (32, 32, 128)
    glob = _hf(num_key_value_heads=4, num_global_key_value_heads=1, head_dim=128, global_head_dim=256)
    assert _detect_head_geometry(glob) == (8, 1, 256)


def test_detect_topology_from_vllm():
    hf = _hf(model_type="gemma4_text", num_hidden_layers=4, layer_types=["sliding_attention", "full_attention"] * 2)
    t = detect_topology_from_vllm(_vllm_config(hf))
    assert (t.model_family, t.num_hidden_layers, t.global_layer_indices) == ("gemma4", 4, (1, 3))
    assert (t.num_query_heads, t.num_kv_heads, t.head_dim) == (8, 1, 256)


def test_detect_topology_unwraps_text_config():
    text = _hf(model_type="llama", num_hidden_layers=2, num_attention_heads=16, num_key_value_heads=4, head_dim=64)
    t = detect_topology_from_vllm(_vllm_config(SimpleNamespace(text_config=text)))
    assert (t.model_family, t.num_hidden_layers, t.num_query_heads) == ("llama", 2, 16)


# ---------------------------------------------------------------- connector

@pytest.mark.parametrize("name,idx", [("model.layers.12.self_attn", 12), ("model.layers.0.self_attn.attn", 0),
                                      ("lm_head", None), ("model.embed_tokens", None)])
def test_parse_layer_index(name, idx):
    assert _parse_layer_index(name) == idx


def test_connector_config_defaults_and_overrides():
    c = KIVConnector(_vllm_config(), role=1)
    assert (c.kiv_config.hot_budget, c.kiv_config.top_p, c.kiv_config.page_size, c.kiv_config.top_pages) == \
        (2048, 256, 128, 32)
    c = KIVConnector(_vllm_config(top_p=128, page_size=64, top_pages=8, hot_budget=512), role=1)
    assert (c.kiv_config.hot_budget, c.kiv_config.top_p, c.kiv_config.page_size, c.kiv_config.top_pages) == \
        (512, 128, 64, 8)
    assert c.role == 1
    assert (c.topology.num_query_heads, c.topology.num_kv_heads, c.topology.head_dim) == (8, 2, 64)


def test_connector_manual_topology():
    topo = dict(global_layer_indices=(1,), independent_kv_layers=(1,), kv_sharing_map={}, num_query_heads=4,
                num_kv_heads=1, head_dim=128, num_hidden_layers=2)
    c = KIVConnector(_vllm_config(topology=topo), role=1)
    assert c.topology.global_layer_indices == (1,) and c.topology.head_dim == 128


def test_connector_is_a_vllm_connector():
    base = pytest.importorskip("vllm.distributed.kv_transfer.kv_connector.v1.base")
    assert issubclass(KIVConnector, base.KVConnectorBase_V1)
    c = KIVConnector(_vllm_config(), role=base.KVConnectorRole.WORKER)
    assert c.role == base.KVConnectorRole.WORKER and not c.has_connector_metadata()


def test_ensure_cold_store_only_for_independent_layers():
    c = KIVConnector(_vllm_config(), role=1)
    assert c._ensure_cold_store(0) is not None and 0 in c.cold_stores
    assert c._ensure_cold_store(0) is c.cold_stores[0]
    c.topology = _topo((0,), (0,))
    assert c._ensure_cold_store(1) is None


def test_get_cold_store_resolves_sharing():
    c = KIVConnector(_vllm_config(), role=1)
    c.topology = _topo((0, 1, 2, 3), (0, 1), {2: 0, 3: 1})
    c._ensure_cold_store(0)
    assert c.get_cold_store(2) is c.cold_stores[0]
    assert c.get_cold_store(3) is None          # source layer 1 has no store yet


@pytest.mark.parametrize("layout", ["slots", "blocks"])
def test_new_rows_are_the_last_slots(layout):
    kv = torch.arange(2 * 12 * 2 * 4, dtype=torch.float32).view(2, 12, 2, 4)
    t = kv if layout == "slots" else kv.view(2, 3, 4, 2, 4)
    k, v = _new_rows(t, 5)
    assert k.shape == (1, 2, 5, 4) and v.shape == (1, 2, 5, 4)
    assert torch.equal(k[0], kv[0, 7:].permute(1, 0, 2)) and torch.equal(v[0], kv[1, 7:].permute(1, 0, 2))
    k, _ = _new_rows(t, 50)                      # more new tokens than slots: all of them
    assert k.shape[2] == 12
    assert _new_rows(torch.zeros(3, 4, 2, 4), 1) is None


def test_save_kv_layer_routes_and_shadows():
    c = KIVConnector(_vllm_config(), role=1)
    c.topology = _topo((0,), (0,))
    st = c.cold_stores[0] = RecordingStore()
    c.save_kv_layer("model.layers.1.self_attn", torch.randn(2, 10, 2, 64),
                    SimpleNamespace(num_decode_tokens=1, num_prefill_tokens=0))
    assert 1 not in c.cold_stores and not st.calls
    kv = torch.randn(2, 5, 2, 64)
    c.save_kv_layer("model.layers.0.self_attn", kv, SimpleNamespace(num_decode_tokens=0, num_prefill_tokens=5))
    assert st.cold_length == 5 and torch.equal(st.calls[0][0][0], kv[0].permute(1, 0, 2))
    c.save_kv_layer("model.layers.0.self_attn", kv, SimpleNamespace(num_decode_tokens=0, num_prefill_tokens=0))
    assert len(st.calls) == 1                    # nothing new: no call
    c.save_kv_layer("model.layers.0.self_attn", torch.zeros(2, 4), SimpleNamespace(num_decode_tokens=1))
    assert len(st.calls) == 1                    # unsupported layout: skipped with a warning


def test_prefill_to_decode_transition_and_step_counter():
    c = KIVConnector(_vllm_config(), role=1)
    c.cold_stores[0] = RecordingStore()
    c.wait_for_save()
    assert c._decode_step == 0 and not c._prefill_complete
    c.save_kv_layer("model.layers.0.self_attn", torch.randn(2, 10, 2, 64),
                    SimpleNamespace(num_decode_tokens=0, num_prefill_tokens=10))
    assert not c._prefill_complete
    c.save_kv_layer("model.layers.0.self_attn", torch.randn(2, 1, 2, 64),
                    SimpleNamespace(num_decode_tokens=1, num_prefill_tokens=0))
    assert c._prefill_complete
    c.wait_for_save()
    c.wait_for_save()
    assert c.decode_step == 2


def test_scheduler_side_defaults_and_shutdown():
    c = KIVConnector(_vllm_config(), role=0)
    assert c.get_num_new_matched_tokens(MagicMock(), 100) == (0, False)
    assert c.update_state_after_alloc(MagicMock(), MagicMock(), 0) is None
    assert c.build_connector_meta(MagicMock()) is not None
    c.register_kv_caches({"model.layers.0.self_attn": torch.zeros(2, 4, 2, 64)})
    assert c._device == torch.device("cpu")
    c._ensure_cold_store(0)
    c.shutdown()
    assert c.cold_stores == {}


# ---------------------------------------------------------------- attention hook

def test_query_reshapes():
    assert hook._query_bhqd(torch.randn(5, 8, 64), 8, 64).shape == (1, 8, 5, 64)
    q2 = torch.randn(3, 512)
    r = hook._query_bhqd(q2, 8, 64)
    assert r.shape == (1, 8, 3, 64) and torch.equal(r[0, 2, 1], q2[1, 128:192])
    assert hook._query_bhqd(torch.randn(1, 8, 1, 64), 8, 64).shape == (1, 8, 1, 64)
    assert hook._query_bhqd(torch.randn(2, 3, 4, 5, 6), 8, 64) is None
    assert hook._query_bhqd(torch.randn(3, 100), 8, 64) is None


def test_output_layouts():
    cold = torch.randn(1, 3, 8, 64)                       # attend's [B, Q, H, D]
    assert torch.equal(hook._as_hot_layout(cold, torch.Size([3, 512])), cold.reshape(3, 512))
    assert torch.equal(hook._as_hot_layout(cold, torch.Size([3, 8, 64])), cold[0])
    assert hook._as_hot_layout(cold, torch.Size([1, 8, 3, 64])).shape == (1, 8, 3, 64)
    assert hook._as_hot_layout(cold, torch.Size([7, 7])) is None


class _Attention(torch.nn.Module):
    """Inner vLLM-style attention: returns a fixed hot output [T, H*D]."""

    def __init__(self, hot):
        super().__init__()
        self.hot = hot

    def forward(self, q, k, v):
        return self.hot


class _SelfAttn(torch.nn.Module):
    def __init__(self, hot):
        super().__init__()
        self.attn = _Attention(hot)


class _Layer(torch.nn.Module):
    def __init__(self, hot):
        super().__init__()
        self.self_attn = _SelfAttn(hot)


def _model(n, hot):
    m = torch.nn.Module()
    m.model = torch.nn.Module()
    m.model.layers = torch.nn.ModuleList([_Layer(hot) for _ in range(n)])
    return m


def test_find_modules():
    hot = torch.zeros(1, 4)
    m = _model(2, hot)
    assert len(hook._find_layers(m)) == 2
    direct = torch.nn.Module()
    direct.layers = torch.nn.ModuleList([_Layer(hot)])
    assert len(hook._find_layers(direct)) == 1
    assert hook._find_layers(torch.nn.Module()) is None
    layer = m.model.layers[0]
    assert hook._find_self_attn(layer) is layer.self_attn
    alt = SimpleNamespace(attention="x")
    assert hook._find_self_attn(alt) == "x" and hook._find_self_attn(SimpleNamespace()) is None
    assert hook._find_inner_attn(layer.self_attn) is layer.self_attn.attn
    same = SimpleNamespace()
    same.attn = same
    assert hook._find_inner_attn(same) is None     # no forward / not an attention class


class _FakeStore:
    def __init__(self, cold_out):
        self.cold_out = cold_out
        self.calls = []

    @property
    def cold_length(self):
        return 1

    def attend(self, q, scaling, cfg, step=-1):
        self.calls.append((tuple(q.shape), scaling, step))
        return self.cold_out


def test_install_merges_hot_and_cold_and_uninstall_restores():
    hot = torch.randn(1, 8 * 64)
    m = _model(4, hot)
    c = KIVConnector(_vllm_config(), role=1)
    c.topology = _topo((0, 2), (0, 2))
    cold = torch.randn(1, 1, 8, 64)
    c.cold_stores[0] = _FakeStore(cold)
    orig = m.model.layers[0].self_attn.attn.forward
    originals = hook.install_attention_hook(m, c)
    assert sorted(originals) == [0, 2]
    q = torch.randn(1, 8 * 64)
    inner = m.model.layers[0].self_attn.attn
    assert torch.equal(inner.forward(q, None, None), hot)            # prefill: hot output only
    c._prefill_complete, c._decode_step = True, 7
    out = inner.forward(q, None, None)
    assert torch.allclose(out, 0.5 * hot + 0.5 * cold.reshape(1, -1), atol=1e-6)
    assert c.cold_stores[0].calls == [((1, 8, 1, 64), 64 ** -0.5, 7)]
    assert torch.equal(m.model.layers[2].self_attn.attn.forward(q, None, None), hot)   # no store yet
    assert torch.equal(m.model.layers[1].self_attn.attn.forward(q, None, None), hot)   # not global
    hook.uninstall_attention_hook(m, originals)
    assert inner.forward == orig


def test_install_without_layers_is_inert():
    c = KIVConnector(_vllm_config(), role=1)
    assert hook.install_attention_hook(torch.nn.Module(), c) == {}


def test_connector_passes_tier_knobs():
    c = KIVConnector(_vllm_config(cold_capacity=131072, host_tokens=1 << 20, stage_pages=512, telemetry=False), role=1)
    cfg = c.kiv_config
    assert (cfg.cold_capacity, cfg.host_tokens, cfg.stage_pages, cfg.telemetry) == (131072, 1 << 20, 512, False)
    with pytest.raises(ValueError):
        KIVConnector(_vllm_config(host_tokens=4096), role=1)   # a host tier needs the HBM ring size
