"""Prefill-shaped retrieval (a chunk of Q positions, G*Q > 32 query rows per KV
head) on the GPU against the oracle: the tcgen05 contraction scorers (coarse:
scores of every query row and page, then the per-row top-k; fine: the max over
all rows of every candidate token by red.max), the candidate select, and the
flash-style tensor-core attention with the causal rule over the hot window.

Shapes cover MHA with head_dim 96 (the c4 Phi-3.5 shape), GQA with several
resident query blocks per CTA and a batch of two (union across the batch),
head_dim 256 (scoring only; its attention runs the split kernel), and a
512-position chunk (two full 256-row blocks, the whole TMEM).  Index sets must
match except ties within 1e-6 relative of the k-th score; attention within
2e-2 relative (bf16/f16 output) of the oracle on the same selection.
"""

import numpy as np
import pytest
import torch

from kiv_b200.synthetic import SynthSpec, make_problem
from oracle.kiv_oracle import causal_hot_mask, eager_attention
from tests.gpu_helpers import DEV, check_selection, oracle_decode, rel_err, run_decode

pytestmark = pytest.mark.gpu

SHAPES = {
    "mha_d96": (SynthSpec(batch=1, num_query_heads=8, num_kv_heads=8, head_dim=96, cold_tokens=60 * 128 + 37,
                          hot_budget=256, query_len=200), dict(top_pages=6, top_p=128)),
    "gqa_b2": (SynthSpec(batch=2, num_query_heads=8, num_kv_heads=2, head_dim=128, cold_tokens=40 * 128 + 5,
                         hot_budget=128, query_len=40), dict(top_pages=4, top_p=64)),
    "mqa_d256": (SynthSpec(batch=1, num_query_heads=4, num_kv_heads=1, head_dim=256, cold_tokens=30 * 128,
                           hot_budget=64, query_len=16), dict(top_pages=4, top_p=64)),
    "mha_q512": (SynthSpec(batch=1, num_query_heads=4, num_kv_heads=4, head_dim=96, cold_tokens=256 * 128 + 64,
                           hot_budget=1024, query_len=512), dict(top_pages=8, top_p=256)),
}
DTYPES = {"bf16": torch.bfloat16, "f16": torch.float16}


@pytest.mark.parametrize("shape,dt", [(s, "bf16") for s in sorted(SHAPES)] + [("mha_d96", "f16")])
def test_prefill_chunk_parity(shape, dt, monkeypatch):
    monkeypatch.delenv("KIV_DISABLE_TCGEN05", raising=False)
    monkeypatch.delenv("KIV_DISABLE_MMA_ATTN", raising=False)
    spec, knobs = SHAPES[shape]
    dtype = DTYPES[dt]
    prob = make_problem(spec, seed=3, dtype=dtype)
    f32 = lambda t: t.float().numpy()
    cfg, cache, store = run_decode(spec, knobs, prob.prefill_k, prob.prefill_v, prob.step_k, prob.step_v,
                                   dtype=dtype)
    ol = oracle_decode(spec, f32(prob.prefill_k), f32(prob.prefill_v), f32(prob.step_k), f32(prob.step_v),
                       storage=dt)
    np.testing.assert_array_equal(store.page_summaries().float().cpu().numpy(), ol.store.summaries)
    q = prob.query.to(DEV)
    scaling = spec.head_dim ** -0.5
    sel, P = store.retrieve_indices(q, scaling, cfg)
    check_selection(store, ol, f32(prob.query), scaling, cfg, sel, P, storage=dt)
    assert store.read_state()[7] == 0, "kernel error bits"
    out = store.attend(q, scaling, cfg, causal=True)
    torch.cuda.synchronize()
    assert store.read_state()[7] == 0, "kernel error bits"
    got = sel[:, :P].cpu().numpy()
    ko, vo = ol.store.gather(got)
    mask = causal_hot_mask(spec.batch, spec.query_len, ol.hot_k.shape[2])
    ref = eager_attention(f32(prob.query), ko, vo, ol.hot_k, ol.hot_v, scaling, mask)
    assert rel_err(out.float().cpu().numpy(), ref) <= 2e-2


def test_prefill_attention_additive_mask_matches_causal_flag():
    """The additive-mask form (no hot-tile skipping) gives the causal flag's output."""
    spec, knobs = SHAPES["mha_d96"]
    prob = make_problem(spec, seed=4, dtype=torch.bfloat16)
    cfg, cache, store = run_decode(spec, knobs, prob.prefill_k, prob.prefill_v, prob.step_k, prob.step_v,
                                   dtype=torch.bfloat16)
    q = prob.query.to(DEV)
    scaling = spec.head_dim ** -0.5
    a = store.attend(q, scaling, cfg, causal=True).float()
    m = torch.from_numpy(causal_hot_mask(1, spec.query_len, store.hot_length)).float().to(DEV)
    b = store.attend(q, scaling, cfg, mask_add=m).float()
    assert torch.equal(a, b)


def test_prefill_tensor_core_and_cuda_core_selections_agree(monkeypatch):
    """Same store and query through the tcgen05 and the CUDA-core scorers."""
    spec, knobs = SHAPES["gqa_b2"]
    prob = make_problem(spec, seed=5, dtype=torch.bfloat16)
    q = prob.query.to(DEV)
    scaling = spec.head_dim ** -0.5
    sels = []
    for disable in (False, True):
        if disable:
            monkeypatch.setenv("KIV_DISABLE_TCGEN05", "1")
        cfg, cache, store = run_decode(spec, knobs, prob.prefill_k, prob.prefill_v, prob.step_k, prob.step_v,
                                       dtype=torch.bfloat16)
        sel, P = store.retrieve_indices(q, scaling, cfg)
        sels.append((sel[:, :P].cpu().numpy(), store))
    (s_tc, st_tc), (s_cc, _) = sels
    # identical up to near-ties: compare as sets per row, allowing a few boundary swaps
    for b in range(spec.batch):
        diff = set(s_tc[b].tolist()) ^ set(s_cc[b].tolist())
        assert len(diff) <= 4, f"row {b}: {len(diff)} differing ids"
