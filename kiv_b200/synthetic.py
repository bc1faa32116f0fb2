"""Seeded synthetic K/V/Q generator shared by the tests, the oracle checks and the bench.

The recipe is the one the benchmark configurations name for KIV's tiered cache
(topic-clustered keys, iid values and queries, one planted needle page):

* keys: the token stream is cut into ``segment``-token topics; every topic and
  KV head draws a centroid from N(0,1)/sqrt(64), and each key is its centroid
  plus N(0, 0.3^2) noise;
* values and queries: iid N(0,1);
* needle: one page-aligned 128-token page inside the cold range whose keys are
  ``2 * q_hat + N(0, 0.3^2)`` per KV head, ``q_hat`` being the unit vector of
  the mean of that KV head's G query heads (of the decode query).

Everything is drawn from one ``torch.Generator`` in a fixed order, in fp32, then
cast to the storage dtype, so a (shape, seed) pair always yields the same
tensors on the same device type.  No public dataset is used: the reference's
own profiling streams FineWeb-Edu text through a real model, which this build
replaces with this generator.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch


@dataclass(frozen=True)
class SynthSpec:
    """Shape of one synthetic single-layer decode problem."""

    batch: int
    num_query_heads: int
    num_kv_heads: int
    head_dim: int
    cold_tokens: int          # tokens that end up in the cold tier after prefill
    hot_budget: int           # tokens kept hot
    page_size: int = 128
    query_len: int = 1        # decode positions per step
    segment: int = 512        # tokens per topic
    needle: bool = True
    centroid_scale: float = 1.0 / math.sqrt(64.0)
    noise: float = 0.3

    @property
    def prefill_tokens(self) -> int:
        return self.cold_tokens + self.hot_budget

    @property
    def groups(self) -> int:
        return self.num_query_heads // self.num_kv_heads


@dataclass
class SynthProblem:
    """Prefill K/V, the decode step's new K/V and its query."""

    spec: SynthSpec
    prefill_k: torch.Tensor   # [B, Hkv, T, D]
    prefill_v: torch.Tensor   # [B, Hkv, T, D]
    step_k: torch.Tensor      # [B, Hkv, Q, D]
    step_v: torch.Tensor      # [B, Hkv, Q, D]
    query: torch.Tensor       # [B, Hq, Q, D]
    needle_page: int          # page index of the planted needle (-1 if none)


def _topic_keys(gen, b, h, t0, n, d, spec, device):
    """Keys for token positions [t0, t0+n) with per-segment centroids."""
    seg = spec.segment
    first = t0 // seg
    last = (t0 + n - 1) // seg
    cent = torch.randn(b, h, last - first + 1, d, generator=gen, device=device) * spec.centroid_scale
    pos = torch.arange(t0, t0 + n, device=device) // seg - first
    keys = cent[:, :, pos, :]
    keys += torch.randn(b, h, n, d, generator=gen, device=device) * spec.noise
    return keys


def make_problem(spec: SynthSpec, seed: int = 0, dtype=torch.float32,
                 device: str | torch.device = "cpu") -> SynthProblem:
    """Draw one problem.  Order of draws: prefill keys, prefill values, query,
    decode-step keys, decode-step values, needle page index, needle noise."""
    device = torch.device(device)
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    B, Hq, Hkv, D = spec.batch, spec.num_query_heads, spec.num_kv_heads, spec.head_dim
    T, Q, S = spec.prefill_tokens, spec.query_len, spec.page_size

    pk = _topic_keys(gen, B, Hkv, 0, T, D, spec, device)
    pv = torch.randn(B, Hkv, T, D, generator=gen, device=device)
    q = torch.randn(B, Hq, Q, D, generator=gen, device=device)
    sk = _topic_keys(gen, B, Hkv, T, Q, D, spec, device)
    sv = torch.randn(B, Hkv, Q, D, generator=gen, device=device)

    needle_page = -1
    full_pages = spec.cold_tokens // S
    if spec.needle and full_pages > 0:
        needle_page = int(torch.randint(0, full_pages, (1,), generator=gen, device=device).item())
        G = spec.groups
        qm = q.float().mean(dim=2).view(B, Hkv, G, D).mean(dim=2)           # [B, Hkv, D]
        qhat = qm / qm.norm(dim=-1, keepdim=True).clamp_min(1e-12)
        noise = torch.randn(B, Hkv, S, D, generator=gen, device=device) * spec.noise
        pk[:, :, needle_page * S:(needle_page + 1) * S, :] = 2.0 * qhat[:, :, None, :] + noise

    cast = lambda x: x.to(dtype)
    return SynthProblem(spec, cast(pk), cast(pv), cast(sk), cast(sv), cast(q), needle_page)


# Shapes of the benchmark configurations (single layer each).
CONFIGS = {
    "c0": SynthSpec(batch=1, num_query_heads=32, num_kv_heads=4, head_dim=64,
                    cold_tokens=65536, hot_budget=2048),
    "c1": SynthSpec(batch=1, num_query_heads=28, num_kv_heads=4, head_dim=128,
                    cold_tokens=131072, hot_budget=2048),
    "c2": SynthSpec(batch=1, num_query_heads=8, num_kv_heads=1, head_dim=256,
                    cold_tokens=1048576, hot_budget=2048),
    "c3": SynthSpec(batch=64, num_query_heads=32, num_kv_heads=8, head_dim=128,
                    cold_tokens=262144, hot_budget=4096),
}

# top_pages / top_p per configuration (page_size is 128 everywhere).
CONFIG_KNOBS = {
    "c0": dict(top_pages=32, top_p=256),
    "c1": dict(top_pages=32, top_p=512),
    "c2": dict(top_pages=64, top_p=1024),
    "c3": dict(top_pages=32, top_p=512),
    "c4": dict(top_pages=32, top_p=256),
}
