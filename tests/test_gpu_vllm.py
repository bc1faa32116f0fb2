"""vLLM integration on the GPU: the connector shadows a layer's prefill and
decode rows out of vLLM-layout cache tensors into a CUDA cold store, and the
attention hook returns ``0.5 * hot + 0.5 * cold`` where ``cold`` is the fused
retrieval attention over the selected cold rows.

Checked against the oracle on the same rows: the cold tier contents (bit
exact), the coarse union and fine selection (stage-wise, ties allowed), and
the merged output (bf16, 2e-2 relative).  A KV-shared layer resolves to its
source layer's store and reuses its selection within the decode step.
"""

from types import SimpleNamespace

import numpy as np
import pytest
import torch

from kiv_b200 import _native as nat
from kiv_b200.vllm import KIVConnector, install_attention_hook, uninstall_attention_hook
from oracle.kiv_oracle import OracleStore, eager_attention
from tests.gpu_helpers import DEV, check_selection, rel_err

pytestmark = pytest.mark.gpu

HQ, HKV, D, PAGE = 8, 2, 128, 128
PREFILL = 20 * PAGE + 37


class _Attention(torch.nn.Module):
    """Inner attention standing in for vLLM's: a fixed hot output [T, Hq*D]."""

    def __init__(self):
        super().__init__()
        self.hot = None

    def forward(self, q, k, v):
        return self.hot


def _model(n_layers):
    m = torch.nn.Module()
    m.model = torch.nn.Module()
    layers = []
    for _ in range(n_layers):
        layer = torch.nn.Module()
        layer.self_attn = torch.nn.Module()
        layer.self_attn.attn = _Attention()
        layers.append(layer)
    m.model.layers = torch.nn.ModuleList(layers)
    return m


def _connector():
    topo = dict(global_layer_indices=(0, 1), independent_kv_layers=(0,), kv_sharing_map={1: 0},
                num_query_heads=HQ, num_kv_heads=HKV, head_dim=D, num_hidden_layers=2)
    cfg = SimpleNamespace(model_config=None,
                          extra_config={"kiv": dict(top_p=256, top_pages=8, page_size=PAGE, topology=topo)})
    c = KIVConnector(cfg, role=1)
    c.register_kv_caches({"model.layers.0.self_attn.attn": torch.zeros(1, device=DEV)})
    return c


def _layout(rows_k, rows_v, layout):
    """vLLM cache tensor holding the rows [T, Hkv, D] (blocks of 16 slots, padded at the front)."""
    kv = torch.stack([rows_k, rows_v])
    if layout == "slots":
        return kv
    T = kv.shape[1]
    pad = (-T) % 16
    kv = torch.cat([torch.zeros(2, pad, HKV, D, dtype=kv.dtype, device=kv.device), kv], 1)
    return kv.view(2, (T + pad) // 16, 16, HKV, D)


@pytest.mark.parametrize("layout", ["slots", "blocks"])
def test_connector_and_hook_match_oracle(layout):
    g = torch.Generator().manual_seed(5)
    k_pre = torch.randn(PREFILL, HKV, D, generator=g)
    v_pre = torch.randn(PREFILL, HKV, D, generator=g)
    k_pre[1500:1510] += 2.0                      # a salient region for the retrieval to find
    k_dec = torch.randn(1, HKV, D, generator=g)
    v_dec = torch.randn(1, HKV, D, generator=g)
    bf = lambda x: x.to(DEV, torch.bfloat16)
    c = _connector()
    model = _model(2)
    originals = install_attention_hook(model, c)
    assert sorted(originals) == [0, 1]

    # prefill, then one decode step; layer 1 reuses layer 0's KV and saves nothing
    c.save_kv_layer("model.layers.0.self_attn.attn", _layout(bf(k_pre), bf(v_pre), layout),
                    SimpleNamespace(num_prefill_tokens=PREFILL, num_decode_tokens=0))
    c.save_kv_layer("model.layers.1.self_attn.attn", _layout(bf(k_pre), bf(v_pre), layout),
                    SimpleNamespace(num_prefill_tokens=PREFILL, num_decode_tokens=0))
    c.wait_for_save()
    c.save_kv_layer("model.layers.0.self_attn.attn", _layout(bf(k_dec), bf(v_dec), layout),
                    SimpleNamespace(num_prefill_tokens=0, num_decode_tokens=1))
    assert list(c.cold_stores) == [0]
    store = c.cold_stores[0]
    assert store.cold_length == PREFILL + 1 and store.hot_length == 0

    ost = OracleStore(1, HKV, D, HQ // HKV, PAGE, "bf16")
    rows = lambda x: x.permute(1, 0, 2).unsqueeze(0).numpy()
    ost.evict_from_hot(rows(k_pre), rows(v_pre))
    ost.evict_from_hot(rows(k_dec), rows(v_dec))
    assert np.array_equal(store.page_summaries().float().cpu().numpy(), ost.summaries), "page summaries"

    q = torch.randn(1, HQ * D, generator=g) + 0.5 * k_pre[1505].repeat_interleave(HQ // HKV, 0).reshape(-1)
    hot = torch.randn(1, HQ * D, generator=g)
    for layer in model.model.layers:
        layer.self_attn.attn.hot = bf(hot)
    outs = [model.model.layers[i].self_attn.attn.forward(bf(q), None, None) for i in (0, 1)]
    c.wait_for_save()
    assert c.decode_step == 1

    qb = bf(q).float().cpu().view(1, HQ, D).permute(1, 0, 2).unsqueeze(0).numpy()
    scaling = D ** -0.5
    sel = store._bufs[("sel", 1, 256, torch.int32)]
    P = int(store.read_state()[nat.ST_SEL])
    assert P == min(256, store.cold_length)
    check_selection(store, SimpleNamespace(store=ost), qb, scaling, c.kiv_config, sel, P, storage="bf16")
    got = sel[:, :P].cpu().numpy()
    ko, vo = ost.gather(got)
    cold = eager_attention(qb, ko, vo, None, None, scaling).reshape(1, HQ * D)
    hot_b = bf(hot).float().cpu().numpy()
    want = 0.5 * hot_b + 0.5 * cold
    for out in outs:
        assert out.shape == (1, HQ * D) and out.dtype == torch.bfloat16
        assert rel_err(out.float().cpu().numpy(), want) <= 2e-2
    uninstall_attention_hook(model, originals)
    assert torch.equal(model.model.layers[0].self_attn.attn.forward(bf(q), None, None), bf(hot))
    c.shutdown()
