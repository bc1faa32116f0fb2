"""bf16 parity of the CUDA path (tcgen05 scoring with the tensor-core attention,
and the CUDA-core scoring and attention) against the oracle run on the same
bf16-valued inputs in float64 math.

Shapes are the c1 (Qwen2.5-7B: Hq 28 / Hkv 4 / D 128), c2 (Gemma-style MQA:
Hq 8 / Hkv 1 / D 256) and c3 (Llama-3-8B, batch of sequences: Hq 32 / Hkv 8 /
D 128, 4 sequences) decode shapes with a reduced cold length.  Index sets
must match except ties within 1e-6 relative of the k-th score (the tensor
cores and the CUDA cores accumulate in fp32 in different orders, the oracle in
float64); attention within 2e-2 relative (bf16 output).
"""

import numpy as np
import pytest
import torch

from kiv_b200.synthetic import SynthSpec, make_problem
from oracle.kiv_oracle import eager_attention
from tests.gpu_helpers import DEV, check_selection, oracle_decode, rel_err, run_decode

pytestmark = pytest.mark.gpu

SHAPES = {
    "c1": (SynthSpec(batch=1, num_query_heads=28, num_kv_heads=4, head_dim=128, cold_tokens=32768,
                     hot_budget=2048), dict(top_pages=32, top_p=512)),
    "c2": (SynthSpec(batch=1, num_query_heads=8, num_kv_heads=1, head_dim=256, cold_tokens=65536,
                     hot_budget=2048), dict(top_pages=64, top_p=1024)),
    # c3 (Llama-3-8B shape, batched decode) with 4 sequences and a shorter cold tier
    "c3": (SynthSpec(batch=4, num_query_heads=32, num_kv_heads=8, head_dim=128, cold_tokens=16384 + 37,
                     hot_budget=1024), dict(top_pages=32, top_p=512)),
    # six sequences (the SMs do not divide evenly over them)
    "c3b6": (SynthSpec(batch=6, num_query_heads=32, num_kv_heads=8, head_dim=128, cold_tokens=8192 + 37,
                       hot_budget=512), dict(top_pages=16, top_p=256)),
}


@pytest.mark.parametrize("path", ["tcgen05", "cuda_cores"])
@pytest.mark.parametrize("shape", sorted(SHAPES))
def test_bf16_decode_parity(shape, path, monkeypatch):
    if path == "cuda_cores":
        monkeypatch.setenv("KIV_DISABLE_TCGEN05", "1")
        monkeypatch.setenv("KIV_DISABLE_MMA_ATTN", "1")
    else:
        monkeypatch.delenv("KIV_DISABLE_TCGEN05", raising=False)
        monkeypatch.delenv("KIV_DISABLE_MMA_ATTN", raising=False)
    spec, knobs = SHAPES[shape]
    prob = make_problem(spec, seed=1, dtype=torch.bfloat16)
    f32 = lambda t: t.float().numpy()
    cfg, cache, store = run_decode(spec, knobs, prob.prefill_k, prob.prefill_v, prob.step_k, prob.step_v,
                                   dtype=torch.bfloat16)
    ol = oracle_decode(spec, f32(prob.prefill_k), f32(prob.prefill_v), f32(prob.step_k), f32(prob.step_v),
                       storage="bf16")
    np.testing.assert_array_equal(store.page_summaries().float().cpu().numpy(), ol.store.summaries)
    q = prob.query.to(DEV)
    scaling = spec.head_dim ** -0.5
    sel, P = store.retrieve_indices(q, scaling, cfg)
    check_selection(store, ol, f32(prob.query), scaling, cfg, sel, P, storage="bf16")
    assert store.read_state()[7] == 0, "kernel error bits"
    # needle page selected
    assert prob.needle_page * spec.page_size in set(sel[0, :P].tolist()) or \
        any(prob.needle_page * 128 <= t < (prob.needle_page + 1) * 128 for t in sel[0, :P].tolist())
    out = store.attend(q, scaling, cfg)
    got = sel[:, :P].cpu().numpy()
    ko, vo = ol.store.gather(got)
    ref = eager_attention(f32(prob.query), ko, vo, ol.hot_k, ol.hot_v, scaling)
    assert rel_err(out.float().cpu().numpy(), ref) <= 2e-2


def test_tcgen05_and_cuda_core_scores_agree(monkeypatch):
    """Same store, both scoring paths: identical selection except near-ties."""
    spec, knobs = SHAPES["c2"]
    prob = make_problem(spec, seed=2, dtype=torch.bfloat16)
    cfg, cache, store = run_decode(spec, knobs, prob.prefill_k, prob.prefill_v, prob.step_k, prob.step_v,
                                   dtype=torch.bfloat16)
    q = prob.query.to(DEV)
    monkeypatch.delenv("KIV_DISABLE_TCGEN05", raising=False)
    s_tc, P = store.retrieve_indices(q, 0.0625, cfg)
    s_tc = set(s_tc[0, :P].tolist())
    monkeypatch.setenv("KIV_DISABLE_TCGEN05", "1")
    s_cc, P2 = store.retrieve_indices(q, 0.0625, cfg)
    s_cc = set(s_cc[0, :P2].tolist())
    assert P == P2
    assert len(s_tc ^ s_cc) <= 4
