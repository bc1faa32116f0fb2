"""Oracle parity at the benchmarked sizes (one layer each).

The bench measures BASELINE's decode configurations at full size; these tests
run the same per-layer shapes through the public surface on the GPU and
compare every stage with the oracle on the same bf16-valued inputs:

* c2 -- Gemma-style MQA (Hq 8 / Hkv 1 / D 256), 1,048,574 cold + 2048 hot
  tokens, top_pages 64, top_p 1024: three eager decode steps (the second one
  completes page 8191, so the coarse pass scores 8192 pages from then on),
  then a captured ``DecodeGraph`` whose capture step and two replays are
  checked the same way;
* c1 -- Qwen2.5-7B shape (Hq 28 / Hkv 4 / D 128), 131,072 cold + 2048 hot,
  top_pages 32, top_p 512: two decode steps;
* c3 slice -- Llama-3-8B shape (Hq 32 / Hkv 8 / D 128), two sequences of
  262,144 cold + 4096 hot tokens each, top_pages 32, top_p 512, the page
  union taken across the batch (kiv/cold_store.py:224): one decode step.

At every step: page summaries bit-exact (c2, c1), coarse union and selected
token sets identical except for ties within 1e-6 relative of the k-th score,
attention within 2e-2 of the float64 oracle over the same selection, both
normwise over the whole output and per query row (the largest absolute error
of a row's D values divided by that row's largest absolute reference value).
"""

import numpy as np
import pytest
import torch

from kiv_b200 import _native as nat
from kiv_b200.decode_graph import DecodeGraph
from kiv_b200.synthetic import SynthSpec, make_problem
from oracle.kiv_oracle import eager_attention
from tests.gpu_helpers import (DEV, check_selection, kernel_union, oracle_decode, rel_err, rel_err_rows,
                               run_decode)

pytestmark = pytest.mark.gpu

BF16_TOL = 2e-2


def _step_rows(spec, n, seed):
    """n decode-step K/V rows: keys near one topic centroid, values N(0,1) (bf16)."""
    g = torch.Generator().manual_seed(seed)
    B, H, D = spec.batch, spec.num_kv_heads, spec.head_dim
    cent = torch.randn(B, H, 1, D, generator=g) / 8.0
    k = cent + 0.3 * torch.randn(B, H, n, D, generator=g)
    v = torch.randn(B, H, n, D, generator=g)
    return k.to(torch.bfloat16), v.to(torch.bfloat16)


def _queries(spec, n, seed, first):
    g = torch.Generator().manual_seed(seed)
    qs = [first] + [torch.randn(spec.batch, spec.num_query_heads, 1, spec.head_dim, generator=g).to(torch.bfloat16)
                    for _ in range(n - 1)]
    return qs


def _check_step(store, ol, q, out, cfg, scaling, what, sel=None, P=None):
    """Selection (union + tokens) and attention parity of the step just run."""
    f32 = q.float().numpy()
    if sel is None:
        sel, P = store.retrieve_indices(q.to(DEV), scaling, cfg)
    check_selection(store, ol, f32, scaling, cfg, sel, P, storage="bf16")
    assert store.read_state()[nat.ST_ERROR] == 0, f"{what}: kernel error bits"
    got = sel[:, :P].cpu().numpy()
    ko, vo = ol.store.gather(got)
    ref = eager_attention(f32, ko, vo, ol.hot_k, ol.hot_v, scaling)
    o = out.float().cpu().numpy().reshape(ref.shape)
    e, er = rel_err(o, ref), rel_err_rows(o, ref)
    assert e <= BF16_TOL and er <= BF16_TOL, f"{what}: attention rel err {e:.3g} (per row {er:.3g})"


def test_c2_full_size_decode_steps_and_graph_replay():
    spec = SynthSpec(batch=1, num_query_heads=8, num_kv_heads=1, head_dim=256, cold_tokens=1048576 - 2,
                     hot_budget=2048)
    knobs = dict(top_pages=64, top_p=1024)
    prob = make_problem(spec, seed=3, dtype=torch.bfloat16)
    n_eager, n_graph = 3, 3
    sk, sv = _step_rows(spec, n_eager + n_graph, seed=31)
    qs = _queries(spec, n_eager + n_graph, seed=32, first=prob.query)
    f32 = lambda t: t.float().numpy()
    cfg, cache, store = run_decode(spec, knobs, prob.prefill_k, prob.prefill_v, sk[:, :, :1], sv[:, :, :1],
                                   dtype=torch.bfloat16, telemetry=False,
                                   cold_capacity=spec.cold_tokens + 4096)
    ol = oracle_decode(spec, f32(prob.prefill_k), f32(prob.prefill_v), f32(sk[:, :, :1]), f32(sv[:, :, :1]),
                       storage="bf16")
    np.testing.assert_array_equal(store.page_summaries().float().cpu().numpy(), ol.store.summaries)
    scaling = spec.head_dim ** -0.5
    completed = False
    for i in range(n_eager):
        if i > 0:
            cache.update(sk[:, :, i:i + 1].to(DEV), sv[:, :, i:i + 1].to(DEV), 0)
            ol.update(f32(sk[:, :, i:i + 1]), f32(sv[:, :, i:i + 1]))
        out = store.attend(qs[i].to(DEV), scaling, cfg, step=cache._decode_step)
        _check_step(store, ol, qs[i], out, cfg, scaling, f"eager step {i}")
        if store.num_pages == 8192:
            completed = True
            np.testing.assert_array_equal(store.page_summaries()[:, :, -1].float().cpu().numpy(),
                                          ol.store.summaries[:, :, -1])
    assert completed and store.cold_length == 1048576 + 1
    # the decode step captured in a CUDA graph: capture runs one step for real
    sq = torch.empty(1, 1, 8, 1, 256, dtype=torch.bfloat16, device=DEV)
    skk = torch.empty(1, 1, 1, 1, 256, dtype=torch.bfloat16, device=DEV)
    svv = torch.empty_like(skk)
    gout = torch.empty(1, 1, 1, 8, 256, dtype=torch.bfloat16, device=DEV)
    graph = None
    for j in range(n_graph):
        i = n_eager + j
        sq.copy_(qs[i].to(DEV)[None])
        skk.copy_(sk[:, :, i:i + 1].to(DEV)[None])
        svv.copy_(sv[:, :, i:i + 1].to(DEV)[None])
        if graph is None:
            graph = DecodeGraph(cache, [0], scaling, sq, skk, svv, gout, max_steps=8)
        else:
            graph.replay()
        torch.cuda.synchronize(DEV)
        ol.update(f32(sk[:, :, i:i + 1]), f32(sv[:, :, i:i + 1]))
        # the graph's own selection: the store's selection buffer and state
        sel = store._buffer("sel", (1, cfg.top_p), torch.int32)
        P = store.read_state()[nat.ST_SEL]
        assert P == cfg.top_p
        _check_step(store, ol, qs[i], gout[0], cfg, scaling, f"graph step {j}", sel=sel, P=P)
    assert store.cold_length == ol.store.cold_length


def test_c1_full_size_decode_steps():
    spec = SynthSpec(batch=1, num_query_heads=28, num_kv_heads=4, head_dim=128, cold_tokens=131072,
                     hot_budget=2048)
    knobs = dict(top_pages=32, top_p=512)
    prob = make_problem(spec, seed=4, dtype=torch.bfloat16)
    f32 = lambda t: t.float().numpy()
    sk, sv = _step_rows(spec, 2, seed=41)
    sk[:, :, :1], sv[:, :, :1] = prob.step_k, prob.step_v
    qs = _queries(spec, 2, seed=42, first=prob.query)
    cfg, cache, store = run_decode(spec, knobs, prob.prefill_k, prob.prefill_v, sk[:, :, :1], sv[:, :, :1],
                                   dtype=torch.bfloat16)
    ol = oracle_decode(spec, f32(prob.prefill_k), f32(prob.prefill_v), f32(sk[:, :, :1]), f32(sv[:, :, :1]),
                       storage="bf16")
    np.testing.assert_array_equal(store.page_summaries().float().cpu().numpy(), ol.store.summaries)
    scaling = spec.head_dim ** -0.5
    for i in range(2):
        if i > 0:
            cache.update(sk[:, :, i:i + 1].to(DEV), sv[:, :, i:i + 1].to(DEV), 0)
            ol.update(f32(sk[:, :, i:i + 1]), f32(sv[:, :, i:i + 1]))
        out = store.attend(qs[i].to(DEV), scaling, cfg, step=cache._decode_step)
        _check_step(store, ol, qs[i], out, cfg, scaling, f"step {i}")
    assert store.cold_length == 131072 + 2


def test_c3_slice_two_sequences_full_length():
    spec = SynthSpec(batch=2, num_query_heads=32, num_kv_heads=8, head_dim=128, cold_tokens=262144,
                     hot_budget=4096)
    knobs = dict(top_pages=32, top_p=512)
    prob = make_problem(spec, seed=5, dtype=torch.bfloat16)
    f32 = lambda t: t.float().numpy()
    cfg, cache, store = run_decode(spec, knobs, prob.prefill_k, prob.prefill_v, prob.step_k, prob.step_v,
                                   dtype=torch.bfloat16)
    ol = oracle_decode(spec, f32(prob.prefill_k), f32(prob.prefill_v), f32(prob.step_k), f32(prob.step_v),
                       storage="bf16")
    del prob.prefill_k, prob.prefill_v
    scaling = spec.head_dim ** -0.5
    out = store.attend(prob.query.to(DEV), scaling, cfg, step=cache._decode_step)
    _check_step(store, ol, prob.query, out, cfg, scaling, "c3 slice")
    # the union is taken across the batch: it holds pages chosen by either sequence
    u = kernel_union(store, 2, 32, 1, cfg)
    assert u.shape[0] > 32 and np.all(np.diff(u) > 0)
