"""End to end through the HF drop-in boundary on a tiny random-init Llama.

With `top_pages` covering every page and `top_p` every cold token, KIV's
retrieval selects the whole cold tier, so attention over [selected cold ;
hot] IS full attention: the KIV-managed model must reproduce the plain
model's logits on the same tokens (bf16 arithmetic, different summation
orders: compared by cosine similarity and top-1 agreement).  Covered:
`KIVMiddleware.install()` / `create_cache()` / `chunked_prefill()` (native
prefill, then eviction to the hot budget), decode steps through the fused
retrieval attention (decode-shaped kernels), and `chunked_retrieval_prefill()`
(every 128-position chunk retrieves from the cold tier: prefill-shaped
kernels with the causal rule from the model's own mask).
"""

import pytest
import torch
from transformers import LlamaConfig, LlamaForCausalLM

from kiv_b200 import KIVConfig, KIVMiddleware
from tests.gpu_helpers import DEV

pytestmark = pytest.mark.gpu


def _model():
    torch.manual_seed(0)
    cfg = LlamaConfig(vocab_size=512, hidden_size=256, intermediate_size=512, num_hidden_layers=2,
                      num_attention_heads=4, num_key_value_heads=2, head_dim=64, max_position_embeddings=4096,
                      attn_implementation="eager")
    return LlamaForCausalLM(cfg).to(DEV, torch.bfloat16).eval()


def _close(a, b):
    a, b = a.float().flatten(), b.float().flatten()
    cos = torch.nn.functional.cosine_similarity(a, b, dim=0).item()
    return cos > 0.999 and int(a.argmax()) == int(b.argmax()), cos


@torch.no_grad()
def test_decode_with_full_selection_matches_full_attention():
    model = _model()
    g = torch.Generator().manual_seed(1)
    ids = torch.randint(0, 512, (1, 900), generator=g).to(DEV)
    mw = KIVMiddleware(model, KIVConfig(hot_budget=128, page_size=128, top_pages=64, top_p=4096, telemetry=False))
    mw.install()
    cache = mw.create_cache()
    logits = mw.chunked_prefill(ids, cache, chunk_size=256)
    store = cache.get_cold_store(0)
    assert store.cold_length == 900 - 128 and store.hot_length == 128
    ok, cos = _close(logits, model_plain_logits(mw, model, ids))
    assert ok, f"prefill logits differ (cos {cos})"
    seq = ids
    for _ in range(3):
        nxt = logits.argmax(-1, keepdim=True)
        seq = torch.cat([seq, nxt], dim=1)
        out = model(input_ids=nxt, past_key_values=cache, use_cache=True)
        logits = out.logits[:, -1]
        ok, cos = _close(logits, model_plain_logits(mw, model, seq))
        assert ok, f"decode logits differ from full attention (cos {cos})"
    assert store.read_state()[7] == 0
    mw.uninstall()


@torch.no_grad()
def test_chunked_retrieval_prefill_matches_full_attention():
    model = _model()
    g = torch.Generator().manual_seed(2)
    ids = torch.randint(0, 512, (1, 1000), generator=g).to(DEV)
    mw = KIVMiddleware(model, KIVConfig(hot_budget=128, page_size=128, top_pages=64, top_p=4096, telemetry=False))
    mw.install()
    cache = mw.create_cache()
    mw.chunked_prefill(ids[:, :600], cache, chunk_size=300)       # native, then evict to the hot budget
    logits = mw.chunked_retrieval_prefill(ids[:, 600:], cache, chunk_size=128)
    store = cache.get_cold_store(0)
    assert store.cold_length + store.hot_length == 1000 and store.cold_length > 0
    ok, cos = _close(logits, model_plain_logits(mw, model, ids))
    assert ok, f"prefill-with-retrieval logits differ from full attention (cos {cos})"
    assert store.read_state()[7] == 0
    mw.uninstall()


def model_plain_logits(mw, model, ids):
    """Last-position logits of the plain model (its own attention, no KIV cache)."""
    impl = mw._resolve_attn_impl()
    mw._set_attn_impl(mw._original_impl)
    try:
        return model(input_ids=ids, use_cache=False).logits[:, -1]
    finally:
        mw._set_attn_impl(impl)
