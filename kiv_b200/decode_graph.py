"""CUDA-graph capture of a whole decode step (all KIV layers) for serving loops.

Every per-step quantity the kernels need (cold length, hot window start and
length, union and selection sizes) lives in device memory, so one decode step
-- per layer: append the new row and evict the oldest, coarse, fine, attention
-- launches the same kernels with the same arguments every time.  This module
captures that step once through the public surface (``TieredKVCache.update``
and ``ColdKVStore.attend``) and replays it; after each replay the host mirrors
of the cache are advanced by the same rule the kernels applied (one row in,
one row out per layer), so the Python view of the cache stays exact.

Preconditions checked at capture: prefill is complete and every layer's hot
window is full (steady state), telemetry is off, and the buffers are reserved
for ``max_steps`` replays, so no replay ever needs a reallocation or a hot
window compaction (both are host decisions).  ``recapture()`` compacts and
captures again when the reserve is used up.
"""

from __future__ import annotations

import torch

from .tiered_cache import TieredKVCache


class DecodeGraph:
    """One captured decode step over ``layers`` of a single-sequence cache."""

    def __init__(self, cache: TieredKVCache, layers: list[int], scaling: float,
                 static_q: torch.Tensor, static_k: torch.Tensor, static_v: torch.Tensor,
                 out: torch.Tensor, max_steps: int, stream: torch.cuda.Stream | None = None):
        """static_q [L, B, Hq, 1, D], static_k/v [L, B, Hkv, 1, D]; out [L, B, 1, Hq, D]."""
        self.cache = cache
        self.layers = list(layers)
        self.scaling = scaling
        self.static_q, self.static_k, self.static_v, self.out = static_q, static_k, static_v, out
        self.max_steps = max_steps
        self.stream = stream or torch.cuda.Stream(cache.device)
        self.graph: torch.cuda.CUDAGraph | None = None
        self.remaining = 0
        self.capture()

    def _check(self) -> None:
        c = self.cache
        if not c._prefill_complete:
            raise RuntimeError("capture a decode step after prefill is complete")
        if c.kiv_config.telemetry:
            raise RuntimeError("telemetry copies are not replay-safe; disable KIVConfig.telemetry")
        for li in self.layers:
            st = c.get_cold_store(li)
            if st.hot_length != c.kiv_config.hot_budget:
                raise RuntimeError("every layer's hot window must be full (steady decode state)")

    def _step(self) -> None:
        cfg = self.cache.kiv_config
        for i, li in enumerate(self.layers):
            self.cache.update(self.static_k[i], self.static_v[i], li)
            st = self.cache.get_cold_store(li)
            st.attend(self.static_q[i], self.scaling, cfg, step=self.cache._decode_step,
                      out=self.out[i])

    def capture(self) -> None:
        self._check()
        c = self.cache
        for li in self.layers:
            st = c.get_cold_store(li)
            # room for the capture step itself plus max_steps replays, no compaction
            st._ensure_hot_room(self.max_steps + 2)
            st.reserve(st.cold_length + self.max_steps + 2,
                       hot_rows=st._hot_start + st.hot_length + self.max_steps + 2)
        # warm the workspaces and buffers outside the capture (this runs one real step)
        self.stream.wait_stream(torch.cuda.current_stream(c.device))
        with torch.cuda.stream(self.stream):
            self._step()
        torch.cuda.current_stream(c.device).wait_stream(self.stream)
        torch.cuda.synchronize(c.device)
        self.graph = torch.cuda.CUDAGraph()
        saved = self._mirror()
        with torch.cuda.graph(self.graph, stream=self.stream):
            self._step()
        # capture recorded the launches but ran nothing: restore the host mirrors
        self._restore(saved)
        self.remaining = self.max_steps

    def _mirror(self):
        c = self.cache
        stores = {li: c.get_cold_store(li) for li in self.layers}
        return (c._decode_step, dict(c._total_tokens),
                {li: (s._cold_len, s._hot_start, s._hot_len, s._cached_step) for li, s in stores.items()})

    def _restore(self, saved) -> None:
        c = self.cache
        c._decode_step, c._total_tokens = saved[0], saved[1]
        for li, (cl, hs, hl, cs) in saved[2].items():
            s = c.get_cold_store(li)
            s._cold_len, s._hot_start, s._hot_len, s._cached_step = cl, hs, hl, cs
            s._invalidate_candidates()

    def replay(self) -> torch.Tensor:
        """Run one captured decode step (inputs read from the static buffers)."""
        if self.remaining <= 0:
            raise RuntimeError("reserve used up: call recapture()")
        self.graph.replay()
        self.remaining -= 1
        c = self.cache
        c._decode_step += 1
        for li in self.layers:
            s = c.get_cold_store(li)
            s._cold_len += 1
            s._hot_start += 1
            s._invalidate_candidates()
            c._total_tokens[li] = s._cold_len + s._hot_len
        return self.out

    def recapture(self) -> None:
        self.graph = None
        self.capture()
