"""Host overflow tier and store persistence on the GPU.

A tiered store keeps only a ring of the newest pages in HBM (here 8 pages),
the older pages in pinned host memory; retrievals stage the union's host pages
(K) and the selected host rows (V) into HBM first.  Every read goes through
copies of the same bytes, so a tiered cache must give BIT-IDENTICAL results to
an HBM-only cache on the same inputs: page summaries, selected token sets,
gathered rows and attention outputs, through prefill, decode steps that cross
page boundaries (ring slots reused, pages spilled), and a prefill-shaped
chunk.  Persistence: a cache saved to disk and loaded into fresh caches (HBM
only, or tiered with another ring size) continues the sequence with the same
outputs as the original.
"""

import numpy as np
import pytest
import torch
from transformers import PretrainedConfig

from kiv_b200 import KIVConfig, ModelTopology, TieredKVCache
from kiv_b200 import _native as nat
from kiv_b200.synthetic import SynthSpec, make_problem
from tests.gpu_helpers import DEV

pytestmark = pytest.mark.gpu

SPEC = SynthSpec(batch=2, num_query_heads=8, num_kv_heads=2, head_dim=128, cold_tokens=40 * 128 + 126,
                 hot_budget=256, query_len=1)
KNOBS = dict(top_pages=4, top_p=128)


def _cache(tiered: bool, ring_pages: int = 8, stage_pages: int = 32, host_pages: int = 64, spec=SPEC):
    extra = {}
    if tiered:
        extra = dict(cold_capacity=ring_pages * 128, host_tokens=host_pages * 128, stage_pages=stage_pages)
    cfg = KIVConfig(hot_budget=spec.hot_budget, page_size=128, telemetry=False, **KNOBS, **extra)
    topo = ModelTopology.manual(global_layer_indices=(0,), independent_kv_layers=(0,), kv_sharing_map={},
                                num_query_heads=spec.num_query_heads, num_kv_heads=spec.num_kv_heads,
                                head_dim=spec.head_dim, num_hidden_layers=1)
    return cfg, TieredKVCache(PretrainedConfig(num_hidden_layers=1), cfg, topo, DEV)


def _steps(n, seed=9, spec=SPEC):
    g = torch.Generator().manual_seed(seed)
    B, Hq, Hkv, D = spec.batch, spec.num_query_heads, spec.num_kv_heads, spec.head_dim
    return [(torch.randn(B, Hq, 1, D, generator=g), 0.3 * torch.randn(B, Hkv, 1, D, generator=g),
             torch.randn(B, Hkv, 1, D, generator=g)) for _ in range(n)]


def _run(cache, cfg, steps, scaling):
    """Decode steps: update + retrieve_indices + attend; returns the per-step results."""
    out = []
    store = cache.get_cold_store(0)
    bf = lambda x: x.to(DEV, torch.bfloat16)
    for q, k, v in steps:
        cache.update(bf(k), bf(v), 0)
        sel, P = store.retrieve_indices(bf(q), scaling, cfg, step=cache._decode_step)
        o = store.attend(bf(q), scaling, cfg, step=cache._decode_step)
        ko, vo = store.retrieve_top_kv(bf(q), scaling, cfg, step=cache._decode_step)
        torch.cuda.synchronize()
        out.append((sel[:, :P].cpu().clone(), o.float().cpu(), ko.float().cpu(), vo.float().cpu()))
    return out


def _prefill(cache, prob):
    bf = lambda x: x.to(DEV, torch.bfloat16)
    cache.update(bf(prob.prefill_k), bf(prob.prefill_v), 0)
    cache.mark_prefill_complete()


def test_tiered_cache_matches_hbm_only_bitwise():
    prob = make_problem(SPEC, seed=4, dtype=torch.bfloat16)
    scaling = SPEC.head_dim ** -0.5
    steps = _steps(5)
    cfg_a, plain = _cache(False)
    cfg_b, tiered = _cache(True)
    _prefill(plain, prob)
    _prefill(tiered, prob)
    sa, sb = plain.get_cold_store(0), tiered.get_cold_store(0)
    assert sb.tiered and sb.cold_length == sa.cold_length == SPEC.cold_tokens
    mem = sb.memory_bytes()
    assert mem["k_index_cpu"] > 0 and mem["v_store_cpu"] == mem["k_index_cpu"]
    assert torch.equal(sa.page_summaries(), sb.page_summaries())
    ra, rb = _run(plain, cfg_a, steps, scaling), _run(tiered, cfg_b, steps, scaling)
    for i, (x, y) in enumerate(zip(ra, rb)):
        assert torch.equal(x[0], y[0]), f"step {i}: selections differ"
        assert torch.equal(x[1], y[1]), f"step {i}: attention outputs differ"
        assert torch.equal(x[2], y[2]) and torch.equal(x[3], y[3]), f"step {i}: gathered rows differ"
    assert torch.equal(sa.page_summaries(), sb.page_summaries())
    assert sb.read_state()[nat.ST_ERROR] == 0 and sa.read_state()[nat.ST_ERROR] == 0
    # the steps crossed a page boundary: a ring slot was reused and its page spilled
    assert sb.cold_length // 128 > SPEC.cold_tokens // 128


def test_tiered_prefill_chunk_matches_hbm_only():
    spec = SynthSpec(batch=1, num_query_heads=8, num_kv_heads=8, head_dim=96, cold_tokens=30 * 128 + 5,
                     hot_budget=128, query_len=96)
    prob = make_problem(spec, seed=6, dtype=torch.bfloat16)
    bf = lambda x: x.to(DEV, torch.bfloat16)
    scaling = spec.head_dim ** -0.5
    outs = []
    for tiered in (False, True):
        cfg, cache = _cache(tiered, ring_pages=6, stage_pages=40, spec=spec)
        _prefill(cache, prob)
        cache.update(bf(prob.step_k), bf(prob.step_v), 0)
        store = cache.get_cold_store(0)
        sel, P = store.retrieve_indices(bf(prob.query), scaling, cfg)
        o = store.attend(bf(prob.query), scaling, cfg, causal=True)
        torch.cuda.synchronize()
        assert store.read_state()[nat.ST_ERROR] == 0
        outs.append((sel[:, :P].cpu(), o.float().cpu()))
    assert torch.equal(outs[0][0], outs[1][0])
    assert torch.equal(outs[0][1], outs[1][1])


def test_stage_capacity_is_reported():
    prob = make_problem(SPEC, seed=4, dtype=torch.bfloat16)
    cfg, cache = _cache(True, stage_pages=1)
    _prefill(cache, prob)
    store = cache.get_cold_store(0)
    q = torch.randn(SPEC.batch, SPEC.num_query_heads, 1, SPEC.head_dim).to(DEV, torch.bfloat16)
    store.attend(q, SPEC.head_dim ** -0.5, cfg)
    torch.cuda.synchronize()
    assert store.read_state()[nat.ST_ERROR] & 16, "a union with more host pages than staging pages must be flagged"


@pytest.mark.parametrize("target", ["hbm", "tiered"])
def test_save_and_resume(tmp_path, target):
    prob = make_problem(SPEC, seed=8, dtype=torch.bfloat16)
    scaling = SPEC.head_dim ** -0.5
    warm, cont = _steps(2, seed=1), _steps(3, seed=2)
    cfg, cache = _cache(True)
    _prefill(cache, prob)
    _run(cache, cfg, warm, scaling)
    cache.save(str(tmp_path / "ckpt"))
    ref = _run(cache, cfg, cont, scaling)
    cfg2, fresh = _cache(target == "tiered", ring_pages=12, stage_pages=24)
    fresh.load(str(tmp_path / "ckpt"))
    s0 = fresh.get_cold_store(0)
    assert s0.cold_length == cache.get_cold_store(0).cold_length - len(cont)
    assert fresh._decode_step == 2 and fresh._prefill_complete
    got = _run(fresh, cfg2, cont, scaling)
    for i, (x, y) in enumerate(zip(ref, got)):
        assert torch.equal(x[0], y[0]), f"step {i}: selections differ after resume"
        assert torch.equal(x[1], y[1]), f"step {i}: outputs differ after resume"


def test_tiered_decode_graph_matches_eager():
    """A captured decode step (spills inside the eviction kernel, staging kernels)
    replays to the same outputs as the eager steps of an identical cache."""
    from kiv_b200.decode_graph import DecodeGraph

    prob = make_problem(SPEC, seed=12, dtype=torch.bfloat16)
    scaling = SPEC.head_dim ** -0.5
    warm, *steps = _steps(7, seed=3)     # capture runs one real step on the static inputs: `warm`
    bf = lambda x: x.to(DEV, torch.bfloat16)
    outs = []
    for graphed in (False, True):
        cfg, cache = _cache(True)
        _prefill(cache, prob)
        store = cache.get_cold_store(0)
        if not graphed:
            for q, k, v in [warm] + steps:
                cache.update(bf(k), bf(v), 0)
                outs.append(store.attend(bf(q), scaling, cfg, step=cache._decode_step).float().cpu())
            outs = outs[1:]
            continue
        sq = bf(warm[0])[None].clone()
        sk = bf(warm[1])[None].clone()
        sv = bf(warm[2])[None].clone()
        out = torch.empty(1, SPEC.batch, 1, SPEC.num_query_heads, SPEC.head_dim, dtype=torch.bfloat16, device=DEV)
        graph = DecodeGraph(cache, [0], scaling, sq, sk, sv, out, max_steps=len(steps) + 2)
        for i, (q, k, v) in enumerate(steps):
            sq[0].copy_(bf(q))
            sk[0].copy_(bf(k))
            sv[0].copy_(bf(v))
            graph.replay()
            torch.cuda.synchronize()
            assert torch.equal(out[0].float().cpu(), outs[i]), f"graph step {i} differs from eager"
        assert store.read_state()[nat.ST_ERROR] == 0
        assert store.cold_length == SPEC.cold_tokens + len(steps) + 1


def test_tiered_steps_and_prefill_chunk_match_oracle():
    """A tiered store (HBM ring of 6 pages, about 1/7 of the cold tier; the rest
    in pinned host memory) against the oracle itself: at each decode step --
    steps that complete a page, so a ring slot is spilled and reused -- the
    page union and token selection equal the oracle's except for ties within
    1e-6 of the k-th score, and the attention is within 2e-2 of the float64
    oracle over the same selection; then a prefill-shaped chunk of 64
    positions (causal over the hot window, union of 1024 query rows staged from
    the host tier) is checked the same way."""
    from oracle.kiv_oracle import OracleLayer, OracleStore, causal_hot_mask, eager_attention
    from tests.gpu_helpers import check_selection, rel_err, rel_err_rows

    prob = make_problem(SPEC, seed=17, dtype=torch.bfloat16)
    cfg, cache = _cache(tiered=True, ring_pages=6, stage_pages=48, host_pages=64)
    _prefill(cache, prob)
    store = cache.get_cold_store(0)
    assert store.tiered
    f32 = lambda t: t.float().numpy()
    ol = OracleLayer(OracleStore(SPEC.batch, SPEC.num_kv_heads, SPEC.head_dim, SPEC.groups, 128, "bf16"),
                     SPEC.hot_budget)
    ol.update(f32(prob.prefill_k), f32(prob.prefill_v))
    ol.mark_prefill_complete()
    scaling = SPEC.head_dim ** -0.5
    bf = lambda x: x.to(DEV, torch.bfloat16)
    pages0 = store.num_pages
    for i, (q, k, v) in enumerate(_steps(4, seed=31)):
        cache.update(bf(k), bf(v), 0)
        ol.update(f32(bf(k).cpu()), f32(bf(v).cpu()))
        qb = bf(q)
        sel, P = store.retrieve_indices(qb, scaling, cfg)
        check_selection(store, ol, f32(qb.cpu()), scaling, cfg, sel, P, storage="bf16")
        out = store.attend(qb, scaling, cfg)
        assert store.read_state()[nat.ST_ERROR] == 0, f"step {i}: kernel error bits"
        ko, vo = ol.store.gather(sel[:, :P].cpu().numpy())
        ref = eager_attention(f32(qb.cpu()), ko, vo, ol.hot_k, ol.hot_v, scaling)
        o = out.float().cpu().numpy()
        assert rel_err(o, ref) <= 2e-2 and rel_err_rows(o, ref) <= 2e-2, f"step {i}"
    assert store.num_pages > pages0, "no page completed during the steps"
    # a prefill-shaped chunk: 64 new positions appended to the hot window (no eviction)
    g = torch.Generator().manual_seed(5)
    Qn = 64
    qc = torch.randn(SPEC.batch, SPEC.num_query_heads, Qn, SPEC.head_dim, generator=g)
    kc = 0.3 * torch.randn(SPEC.batch, SPEC.num_kv_heads, Qn, SPEC.head_dim, generator=g)
    vc = torch.randn(SPEC.batch, SPEC.num_kv_heads, Qn, SPEC.head_dim, generator=g)
    cache._prefill_complete = False
    cache.update(bf(kc), bf(vc), 0)
    ol.prefill_complete = False
    ol.update(f32(bf(kc).cpu()), f32(bf(vc).cpu()))
    qb = bf(qc)
    sel, P = store.retrieve_indices(qb, scaling, cfg)
    check_selection(store, ol, f32(qb.cpu()), scaling, cfg, sel, P, storage="bf16")
    out = store.attend(qb, scaling, cfg, causal=True)
    assert store.read_state()[nat.ST_ERROR] == 0, "prefill chunk: kernel error bits"
    ko, vo = ol.store.gather(sel[:, :P].cpu().numpy())
    hot = ol.hot_k.shape[2]
    ref = eager_attention(f32(qb.cpu()), ko, vo, ol.hot_k, ol.hot_v, scaling,
                          hot_mask=causal_hot_mask(SPEC.batch, Qn, hot))
    o = out.float().cpu().numpy()
    assert rel_err(o, ref) <= 2e-2 and rel_err_rows(o, ref) <= 2e-2, "prefill chunk"
