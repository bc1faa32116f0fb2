"""Generate the golden fixtures in this folder by running the REFERENCE implementation.

Run in a container where the reference project is importable:

    python tests/golden/make_golden.py --reference <path to the reference checkout>

It imports the reference package ``kiv`` (``TieredKVCache``, ``ColdKVStore``,
``KIVConfig``, ``ModelTopology``) and HF's ``eager_attention_forward`` (the
attention the reference wrapper calls with the default ``eager`` implementation),
drives one decode layer-step per case on CPU in fp32, and records the
reference's decisions: the coarse page union and the selected token ids (both
read from the reference's own retrieval telemetry), the returned K/V, the page
summaries and the attention output over ``[cold ; hot]``.

Inputs come from ``kiv_b200.synthetic.make_problem`` (seeded), so the large
``c0`` case stores only outputs; the tests regenerate its inputs from the seed.
Small cases store their inputs as well.
"""

from __future__ import annotations

import argparse
import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)

from kiv_b200.synthetic import SynthSpec, make_problem  # noqa: E402

# name -> (spec kwargs, knobs, flow)
CASES = {
    "gqa_basic": (dict(batch=1, num_query_heads=4, num_kv_heads=2, head_dim=16,
                       cold_tokens=200, hot_budget=24, page_size=8, segment=32),
                  dict(top_pages=4, top_p=12), "decode"),
    "batch2_union": (dict(batch=2, num_query_heads=4, num_kv_heads=2, head_dim=8,
                          cold_tokens=160, hot_budget=16, page_size=8, segment=32),
                     dict(top_pages=3, top_p=10), "decode"),
    "mqa": (dict(batch=1, num_query_heads=8, num_kv_heads=1, head_dim=32,
                 cold_tokens=512, hot_budget=32, page_size=16, segment=64),
            dict(top_pages=5, top_p=40), "decode"),
    "mha_q3": (dict(batch=1, num_query_heads=3, num_kv_heads=3, head_dim=12,
                    cold_tokens=96, hot_budget=20, page_size=8, segment=16, query_len=3),
               dict(top_pages=2, top_p=9), "decode"),
    "partial_only": (dict(batch=1, num_query_heads=4, num_kv_heads=2, head_dim=8,
                          cold_tokens=5, hot_budget=12, page_size=8, segment=16),
                     dict(top_pages=2, top_p=4), "decode"),
    "np_lt_top_pages": (dict(batch=1, num_query_heads=4, num_kv_heads=1, head_dim=8,
                             cold_tokens=27, hot_budget=8, page_size=8, segment=16),
                        dict(top_pages=6, top_p=5), "decode"),
    "p_gt_candidates": (dict(batch=1, num_query_heads=2, num_kv_heads=1, head_dim=8,
                             cold_tokens=123, hot_budget=8, page_size=8, segment=16),
                        dict(top_pages=2, top_p=100), "decode"),
    "page_boundary": (dict(batch=1, num_query_heads=4, num_kv_heads=2, head_dim=8,
                           cold_tokens=63, hot_budget=10, page_size=8, segment=16),
                      dict(top_pages=3, top_p=7), "decode"),
    "shared_reuse": (dict(batch=1, num_query_heads=4, num_kv_heads=2, head_dim=16,
                          cold_tokens=256, hot_budget=16, page_size=8, segment=32),
                     dict(top_pages=3, top_p=10), "reuse"),
    "c0": (dict(batch=1, num_query_heads=32, num_kv_heads=4, head_dim=64,
                cold_tokens=65536, hot_budget=2048, page_size=128, segment=512),
           dict(top_pages=32, top_p=256), "decode"),
}

SMALL_LIMIT = 1 << 16   # store inputs when prefill K has at most this many elements


def _stub_module(groups):
    class _M(torch.nn.Module):
        pass
    m = _M()
    m.num_key_value_groups = groups
    m.training = False
    return m


def run_case(name, ref_kiv, eager):
    spec_kw, knobs, flow = CASES[name]
    spec = SynthSpec(**spec_kw)
    prob = make_problem(spec, seed=0, dtype=torch.float32)
    KIVConfig = ref_kiv["KIVConfig"]
    ModelTopology = ref_kiv["ModelTopology"]
    TieredKVCache = ref_kiv["TieredKVCache"]
    from transformers import PretrainedConfig

    cfg = KIVConfig(hot_budget=spec.hot_budget, page_size=spec.page_size,
                    prefetch_stream=False, **knobs)
    shared = flow == "reuse"
    topo = ModelTopology.manual(
        global_layer_indices=(0, 1) if shared else (0,),
        independent_kv_layers=(0,),
        kv_sharing_map={1: 0} if shared else {},
        num_query_heads=spec.num_query_heads, num_kv_heads=spec.num_kv_heads,
        head_dim=spec.head_dim, num_hidden_layers=2 if shared else 1)
    cache = TieredKVCache(PretrainedConfig(num_hidden_layers=2 if shared else 1),
                          cfg, topo, torch.device("cpu"))
    cache.update(prob.prefill_k, prob.prefill_v, 0)
    cache.mark_prefill_complete()
    keys, values = cache.update(prob.step_k, prob.step_v, 0)
    store = cache.get_cold_store(0)
    scaling = spec.head_dim ** -0.5
    queries = [prob.query]
    if shared:
        g = torch.Generator().manual_seed(1)
        queries.append(torch.randn(prob.query.shape, generator=g))
    out = {}
    for li, q in enumerate(queries):
        ck, cv = store.retrieve_top_kv(q, scaling, cfg, step=cache._decode_step)
        hot_len = keys.shape[2]
        Q = q.shape[2]
        mask = None
        if Q > 1:
            i = torch.arange(Q)[:, None]
            j = torch.arange(hot_len)[None, :]
            mask = torch.where(j <= hot_len - Q + i, 0.0, float("-inf"))
            mask = mask.expand(spec.batch, 1, Q, hot_len)
            mask = ref_kiv["extend_mask_for_cold"](mask, ck.shape[2])
        K = torch.cat([ck, keys], dim=2)
        V = torch.cat([cv, values], dim=2)
        attn, _ = eager(_stub_module(spec.groups), q, K, V, mask, scaling=scaling, dropout=0.0)
        out[f"attn_{li}"] = attn.numpy()
        out[f"k_out_{li}"] = ck.numpy()
        out[f"v_out_{li}"] = cv.numpy()
    snap = store.telemetry_snapshot()
    recs = snap["recent"]
    coarse = [r for r in recs if r["kind"] == "coarse"]
    fine = [r for r in recs if r["kind"] == "fine"]
    for li in range(len(queries)):
        out[f"union_{li}"] = np.asarray(coarse[li]["pages_selected"], np.int64)
        out[f"coarse_skipped_{li}"] = np.asarray(coarse[li]["skipped"])
        out[f"selected_{li}"] = np.asarray(fine[li]["selected_token_indices"], np.int64)
        out[f"actual_P_{li}"] = np.asarray(fine[li]["actual_P"])
    store._materialize()
    summ = store._page_summaries
    out["summaries"] = (summ.numpy() if summ is not None
                        else np.zeros((spec.batch, spec.num_kv_heads, 0, spec.head_dim), np.float32))
    out["cold_length"] = np.asarray(store.cold_length)
    out["num_pages"] = np.asarray(store.num_pages)
    out["hot_len"] = np.asarray(keys.shape[2])
    if prob.prefill_k.numel() <= SMALL_LIMIT:
        out["prefill_k"] = prob.prefill_k.numpy()
        out["prefill_v"] = prob.prefill_v.numpy()
        out["step_k"] = prob.step_k.numpy()
        out["step_v"] = prob.step_v.numpy()
        for li, q in enumerate(queries):
            out[f"query_{li}"] = q.numpy()
    meta = dict(spec=spec_kw, knobs=knobs, flow=flow, seed=0, scaling=scaling,
                queries=len(queries), needle_page=prob.needle_page)
    out["meta"] = np.asarray(json.dumps(meta))
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path of the reference checkout")
    ap.add_argument("--only", default=None)
    args = ap.parse_args()
    sys.path.insert(0, os.path.abspath(args.reference))
    from kiv.config import KIVConfig
    from kiv.model_topology import ModelTopology
    from kiv.tiered_cache import TieredKVCache
    from kiv.mask_utils import extend_mask_for_cold
    from transformers.models.llama.modeling_llama import eager_attention_forward
    ref = dict(KIVConfig=KIVConfig, ModelTopology=ModelTopology, TieredKVCache=TieredKVCache,
               extend_mask_for_cold=extend_mask_for_cold)
    torch.set_num_threads(os.cpu_count() or 1)
    for name in CASES:
        if args.only and name != args.only:
            continue
        out = run_case(name, ref, eager_attention_forward)
        path = os.path.join(HERE, f"{name}.npz")
        np.savez_compressed(path, **out)
        print(f"{name}: cold={int(out['cold_length'])} pages={int(out['num_pages'])} "
              f"U={out['union_0'].shape[0]} P={int(out['actual_P_0'])} -> {os.path.basename(path)}")


if __name__ == "__main__":
    main()
