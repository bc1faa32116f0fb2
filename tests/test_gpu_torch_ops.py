"""A decode layer-step through ``torch.ops.kiv.*``, eager and inside a
``torch.cuda.graph`` capture, against the oracle.

The store's buffers come from the public surface (prefill + mark complete);
then every kernel of the step is called as a PyTorch operator on those
tensors: append_evict (new row in, oldest hot row to the cold tier),
coarse_select, fine_select and attend.  The first step runs eagerly, the next
two are replays of a captured graph of the same four operators with their
inputs copied into static buffers.  After each step the page union and the
selected token set must equal the oracle's except for ties within 1e-6 of the
k-th score, and the attention output must be within 2e-2 of the float64
oracle over the same selection (bf16 store).
"""

import numpy as np
import pytest
import torch

from kiv_b200 import _native as nat
from kiv_b200 import ops
from kiv_b200.synthetic import SynthSpec, make_problem
from oracle.kiv_oracle import OracleLayer, OracleStore, eager_attention, topk_set_mismatch
from tests.gpu_helpers import DEV, coarse_union_mismatch, make_cache, rel_err, rel_err_rows

pytestmark = pytest.mark.gpu


def test_decode_step_through_torch_ops_eager_and_graph():
    spec = SynthSpec(batch=1, num_query_heads=8, num_kv_heads=2, head_dim=128, cold_tokens=20000 + 61,
                     hot_budget=512)
    knobs = dict(top_pages=8, top_p=256)
    prob = make_problem(spec, seed=21, dtype=torch.bfloat16)
    f32 = lambda t: t.float().numpy()
    # prefill through the public surface; the decode steps below go through the operators only
    cfg, cache = make_cache(spec, knobs, telemetry=False)
    cache.update(prob.prefill_k.to(DEV), prob.prefill_v.to(DEV), 0)
    cache.mark_prefill_complete()
    store = cache.get_cold_store(0)
    ol = OracleLayer(OracleStore(1, 2, 128, 4, 128, "bf16"), spec.hot_budget)
    ol.update(f32(prob.prefill_k), f32(prob.prefill_v))
    ol.mark_prefill_complete()
    store._ensure_hot_room(8)
    store.reserve(store.cold_length + 8, hot_rows=store._hot_start + store.hot_length + 8)
    K = ops.kiv()
    so, geom = store._op_store(hot_hint=spec.hot_budget)
    g = torch.Generator().manual_seed(22)
    steps = [(torch.randn(1, 8, 1, 128, generator=g), 0.1 * torch.randn(1, 2, 1, 128, generator=g),
              torch.randn(1, 2, 1, 128, generator=g)) for _ in range(3)]
    steps[0] = (prob.query.float(), steps[0][1], steps[0][2])
    bf = lambda t: t.to(DEV, torch.bfloat16)
    q_s, k_s, v_s = bf(steps[0][0]), bf(steps[0][1]), bf(steps[0][2])
    scaling = 128 ** -0.5
    lay = K.workspace_layout(so, geom, q_s, cfg.top_pages, cfg.top_p)
    ws = torch.zeros(lay[10] + 256, dtype=torch.uint8, device=DEV)
    ws = ws[(-ws.data_ptr()) % 256:][:lay[10]]
    sel = torch.zeros(1, cfg.top_p, dtype=torch.int32, device=DEV)
    out = torch.zeros(1, 1, 8, 128, dtype=torch.bfloat16, device=DEV)
    state = so[5]

    def step():
        K.append_evict(so, geom, k_s, v_s, spec.hot_budget, 1)
        K.coarse_select(so, geom, q_s, scaling, cfg.top_pages, cfg.top_p, 0.0, ws, None, None)
        K.fine_select(so, geom, q_s, scaling, cfg.top_pages, cfg.top_p, 0.0, ws, sel, None)
        K.attend(so, geom, q_s, scaling, cfg.top_pages, cfg.top_p, 0.0, ws, sel, None, False, 0, 1, out, None)

    def check(i):
        qn, kn, vn = (bf(x).float().cpu().numpy() for x in steps[i])
        ol.update(kn, vn)
        words = state.cpu().tolist()
        assert words[nat.ST_ERROR] == 0, f"step {i}: kernel error bits"
        assert words[nat.ST_COLD_LEN] == ol.store.cold_length
        U, P = words[nat.ST_UNION], words[nat.ST_SEL]
        union = ws[lay[2]:lay[2] + 4 * U].view(torch.int32).cpu().numpy().astype(np.int64)
        union_ref, _, sc = ol.store.coarse(qn, scaling, cfg.top_pages)
        assert coarse_union_mismatch(union, union_ref, sc, min(cfg.top_pages, ol.store.num_pages)) == []
        cand = ol.store.candidates(union)
        agg, sel_ref = ol.store.fine(qn, scaling, cand, cfg.top_p)
        assert P == sel_ref.shape[1]
        got = sel[0, :P].cpu().numpy().astype(np.int64)
        pos = {int(t): j for j, t in enumerate(cand)}
        assert topk_set_mismatch(got, sel_ref[0], lambda t: agg[0, pos[t]], P, agg[0]) == [], f"step {i}"
        ko, vo = ol.store.gather(got[None])
        ref = eager_attention(qn, ko, vo, ol.hot_k, ol.hot_v, scaling)
        o = out.float().cpu().numpy()
        assert rel_err(o, ref) <= 2e-2 and rel_err_rows(o, ref) <= 2e-2, f"step {i}"

    stream = torch.cuda.Stream(DEV)
    stream.wait_stream(torch.cuda.current_stream(DEV))
    with torch.cuda.stream(stream):
        step()                        # eager step 0
    torch.cuda.current_stream(DEV).wait_stream(stream)
    torch.cuda.synchronize(DEV)
    check(0)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        step()                        # captured, not run
    for i in (1, 2):
        q_s.copy_(bf(steps[i][0]))
        k_s.copy_(bf(steps[i][1]))
        v_s.copy_(bf(steps[i][2]))
        graph.replay()
        torch.cuda.synchronize(DEV)
        check(i)
