"""Shared helpers of the GPU tests: run a decode layer-step through the public
surface on CUDA, and compare each stage with the oracle on the same inputs."""

from __future__ import annotations

import numpy as np
import torch
from transformers import PretrainedConfig

from kiv_b200 import KIVConfig, ModelTopology, TieredKVCache
from kiv_b200 import _native as nat
from oracle.kiv_oracle import (OracleLayer, OracleStore, eager_attention, to_storage,
                               topk_set_mismatch, topk_total_order)

DEV = torch.device("cuda:0") if torch.cuda.is_available() else None
STORAGE = {torch.float32: "f32", torch.bfloat16: "bf16", torch.float16: "f16"}


def make_cache(spec, knobs, dtype=torch.float32, shared=False, **cfg_extra):
    cfg = KIVConfig(hot_budget=spec.hot_budget, page_size=spec.page_size, **knobs, **cfg_extra)
    topo = ModelTopology.manual(
        global_layer_indices=(0, 1) if shared else (0,), independent_kv_layers=(0,),
        kv_sharing_map={1: 0} if shared else {}, num_query_heads=spec.num_query_heads,
        num_kv_heads=spec.num_kv_heads, head_dim=spec.head_dim,
        num_hidden_layers=2 if shared else 1)
    cache = TieredKVCache(PretrainedConfig(num_hidden_layers=2 if shared else 1), cfg, topo, DEV)
    return cfg, cache


def run_decode(spec, knobs, prefill_k, prefill_v, step_k, step_v, dtype=torch.float32, shared=False,
               **cfg_extra):
    """Prefill + mark complete + one decode update; returns (cfg, cache, store)."""
    cfg, cache = make_cache(spec, knobs, dtype, shared, **cfg_extra)
    t = lambda x: torch.as_tensor(x).to(DEV, dtype)
    cache.update(t(prefill_k), t(prefill_v), 0)
    cache.mark_prefill_complete()
    cache.update(t(step_k), t(step_v), 0)
    return cfg, cache, cache.get_cold_store(0)


def oracle_decode(spec, prefill_k, prefill_v, step_k, step_v, storage="f32"):
    ost = OracleStore(spec.batch, spec.num_kv_heads, spec.head_dim, spec.groups, spec.page_size, storage)
    ol = OracleLayer(ost, spec.hot_budget)
    ol.update(np.asarray(prefill_k, np.float32), np.asarray(prefill_v, np.float32))
    ol.mark_prefill_complete()
    ol.update(np.asarray(step_k, np.float32), np.asarray(step_v, np.float32))
    return ol


def workspace_view(store, B, Hq, Q, cfg):
    """(ws tensor, layout) of the workspace used for this query shape."""
    key = (B, Hq, Q, cfg.top_pages, cfg.top_p)
    ws, lay = store._ws[key]
    return ws, lay


def kernel_union(store, B, Hq, Q, cfg):
    ws, lay = workspace_view(store, B, Hq, Q, cfg)
    u = store.read_state()[nat.ST_UNION]
    return ws[lay[2]:lay[2] + 4 * lay[8]].view(torch.int32)[:u].cpu().numpy().astype(np.int64)


def coarse_union_mismatch(union_got, union_ref, coarse_scores, k, rtol=1e-6):
    """Pages in the union difference that are not within rtol of some row's k-th score."""
    diff = set(union_got.tolist()) ^ set(union_ref.tolist())
    if not diff:
        return []
    rows = coarse_scores.reshape(-1, coarse_scores.shape[-1])
    bounds = np.sort(rows, axis=1)[:, ::-1][:, k - 1]
    return [p for p in diff
            if not (np.abs(rows[:, p] - bounds) <= rtol * np.maximum(np.abs(bounds), 1e-30)).any()]


def check_selection(store, ol, query, scaling, cfg, sel, P, storage="f32", rtol=1e-6,
                    check_coarse=True):
    """Stage-wise selection parity.  Returns the oracle fine result on the kernel's union.

    ``check_coarse=False`` for a call that reused an earlier call's union."""
    B, Hq, Q, _ = query.shape
    q = np.asarray(query, np.float32)
    ost = ol.store
    if ost.num_pages > 0 and not check_coarse:
        union_got = kernel_union(store, B, Hq, Q, cfg)
    elif ost.num_pages > 0:
        union_ref, top, sc = ost.coarse(q, scaling, cfg.top_pages)
        union_got = kernel_union(store, B, Hq, Q, cfg)
        k = min(cfg.top_pages, ost.num_pages)
        bad = coarse_union_mismatch(union_got, union_ref, sc, k, rtol)
        assert bad == [], f"coarse union mismatch beyond ties: {bad[:5]}"
    else:
        union_got = np.zeros((0,), np.int64)
    cand = ost.candidates(union_got)
    agg, sel_ref = ost.fine(q, scaling, cand, cfg.top_p)
    assert P == sel_ref.shape[1], (P, sel_ref.shape)
    pos = {int(t): i for i, t in enumerate(cand)}
    got = sel[:, :P].cpu().numpy()
    for b in range(B):
        assert np.all(np.diff(got[b]) > 0), "selected ids must be ascending and unique"
        bad = topk_set_mismatch(got[b], sel_ref[b], lambda t: agg[b, pos[t]], P, agg[b], rtol)
        assert bad == [], f"fine selection mismatch (batch {b}) beyond ties: {bad[:5]}"
    return cand, agg, sel_ref


def rel_err(a, b):
    """Normwise relative error: the largest absolute difference over the whole
    output divided by the largest absolute reference value (see also
    ``rel_err_rows`` for the same ratio per query row)."""
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


def rel_err_rows(a, b):
    """Largest per-row relative error: for every query row (the last axis holds
    its D values), the largest absolute difference divided by that row's
    largest absolute reference value; the maximum over rows."""
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    num = np.abs(a - b).max(axis=-1)
    den = np.maximum(np.abs(b).max(axis=-1), 1e-30)
    return float((num / den).max())
