"""CPU oracle for KIV's tiered-cache retrieval path -- TEST INFRASTRUCTURE ONLY.

This module restates, in numpy, the algorithm of the reference's cold store and
attention wrapper.  It exists to check the CUDA path: only ``tests/``,
``__graft_entry__.smoke()`` and the ``cpu_baseline`` / ``--impl reference`` legs
of ``bench.py`` may import it, and never as the thing that is measured or
shipped.  The product path (``kiv_b200``) never imports it.

Parity pin: the oracle is checked against golden vectors produced by running the
reference implementation itself (``tests/golden/make_golden.py`` imports the
reference package and writes ``tests/golden/*.npz``; ``tests/test_oracle_golden.py``
compares).  Reference files cited below are paths inside the reference project.

Numerics (chosen so that the CUDA kernels can be compared exactly where the
math allows it):

* page summary (kiv/cold_store.py:160-165 ``page_k.mean(dim=2)``): fp32 sum of
  the 128 page rows in token order, divided by the page size, rounded to the
  storage dtype.  The CUDA eviction kernel does the same fp32 operations in the
  same order, so summaries compare bit-exactly.
* scores (kiv/cold_store.py:205-208 coarse, :332-335 fine): float64 dot products
  of the storage-valued query and keys, times ``scaling``.  The reference
  computes them in the storage dtype; index parity is asserted with a 1e-6
  relative tie band around the k-th score.
* top-k (kiv/cold_store.py:212, :341 ``torch.topk``): the k largest under the
  total order (score descending, index ascending).  ``torch.topk`` leaves tie
  order unspecified; this order is the one the CUDA select kernels implement.
* the selected cold tokens are reported in ascending global token order (the
  reference returns them in descending-score order; attention over them does
  not depend on the order).
"""

from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

STORAGE_DTYPES = ("f32", "bf16", "f16")


# --------------------------------------------------------------------------
# storage rounding
# --------------------------------------------------------------------------

def round_bf16(x: np.ndarray) -> np.ndarray:
    """Round float32 values to bfloat16 (round-to-nearest-even), returned as float32."""
    a = np.ascontiguousarray(x, dtype=np.float32)
    u = a.view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    return u.astype(np.uint32).view(np.float32).reshape(a.shape)


def to_storage(x: np.ndarray, storage: str) -> np.ndarray:
    """Round to the storage dtype and return float32 holding those values."""
    x = np.asarray(x, dtype=np.float32)
    if storage == "f32":
        return x.copy()
    if storage == "bf16":
        return round_bf16(x)
    if storage == "f16":
        return x.astype(np.float16).astype(np.float32)
    raise ValueError(f"unknown storage dtype {storage!r}")


# --------------------------------------------------------------------------
# ordering helpers
# --------------------------------------------------------------------------

def topk_total_order(scores: np.ndarray, k: int) -> np.ndarray:
    """Indices of the k largest entries of a 1-D array, ties broken by lowest index.

    Restates ``torch.topk(k)`` (kiv/cold_store.py:212, :341) with a fixed tie rule.
    """
    n = scores.shape[0]
    k = min(k, n)
    s = scores.astype(np.float64, copy=False)
    if k < n:
        part = np.argpartition(-s, k - 1)[:k]
        cand = np.nonzero(s >= s[part].min())[0]     # every key tied with the k-th
    else:
        cand = np.arange(n)
    order = cand[np.lexsort((cand, -s[cand]))]
    return order[:k]


def page_summary(page_rows: np.ndarray, storage: str) -> np.ndarray:
    """Mean of the rows of one page: ``[..., S, D] -> [..., D]``.

    kiv/cold_store.py:164.  fp32 sum in token order, then divide, then round.
    """
    S = page_rows.shape[-2]
    acc = np.zeros(page_rows.shape[:-2] + page_rows.shape[-1:], dtype=np.float32)
    for t in range(S):
        acc += page_rows[..., t, :].astype(np.float32)
    return to_storage(acc / np.float32(S), storage)


def _group_rows(query: np.ndarray, hkv: int) -> np.ndarray:
    """[B, Hq, Q, D] -> [B, Hkv, G*Q, D] in (head-in-group, position) row order."""
    B, Hq, Q, D = query.shape
    G = Hq // hkv
    return query.reshape(B, hkv, G, Q, D).reshape(B, hkv, G * Q, D)


# --------------------------------------------------------------------------
# the cold store
# --------------------------------------------------------------------------

@dataclass
class RetrievalResult:
    """Everything one ``retrieve_top_kv`` call decides."""

    union_pages: np.ndarray          # [U] sorted page ids (empty if coarse skipped)
    row_top_pages: np.ndarray | None  # [B, Hq, Q, k] per-row top pages (score order)
    coarse_scores: np.ndarray | None  # [B, Hq, Q, Np] float64
    cand_idx: np.ndarray             # [C] global token id per candidate position
    agg_scores: np.ndarray           # [B, C] float64, max over heads and positions
    selected: np.ndarray             # [B, P] global token ids, ascending
    k_out: np.ndarray                # [B, Hkv, P, D]
    v_out: np.ndarray                # [B, Hkv, P, D]
    coarse_skipped: bool


@dataclass
class OracleStore:
    """Restates ``ColdKVStore`` (kiv/cold_store.py:35-371) on numpy arrays.

    Tokens are kept in one token-indexed array per tensor (finalized pages and
    the partial page together); page summaries are kept per finalized page.
    """

    batch: int
    num_kv_heads: int
    head_dim: int
    groups: int
    page_size: int
    storage: str = "f32"
    compute: type = np.float64          # score arithmetic (float64: parity; float32: timing)
    cached_step: int = field(default=-1, init=False)
    cached_union: np.ndarray | None = field(default=None, init=False)
    cached_batch: int = field(default=-1, init=False)

    def __post_init__(self):
        shape = (self.batch, self.num_kv_heads, 16, self.head_dim)
        self._k = np.zeros(shape, np.float32)
        self._v = np.zeros(shape, np.float32)
        self._s = np.zeros(shape, np.float32)
        self._n = 0

    # token-indexed views (storage grows by doubling: appends are amortized O(1))
    @property
    def k(self) -> np.ndarray:
        return self._k[:, :, :self._n]

    @property
    def v(self) -> np.ndarray:
        return self._v[:, :, :self._n]

    @property
    def summaries(self) -> np.ndarray:
        return self._s[:, :, :self.num_pages]

    def _grow(self, need: int) -> None:
        cap = self._k.shape[2]
        if need <= cap:
            return
        cap = max(need, 2 * cap)
        for name in ("_k", "_v"):
            old = getattr(self, name)
            new = np.zeros(old.shape[:2] + (cap,) + old.shape[3:], np.float32)
            new[:, :, :self._n] = old[:, :, :self._n]
            setattr(self, name, new)
        pages = cap // self.page_size + 1
        if pages > self._s.shape[2]:
            new = np.zeros(self._s.shape[:2] + (pages,) + self._s.shape[3:], np.float32)
            new[:, :, :self.num_pages] = self._s[:, :, :self.num_pages]
            self._s = new

    # -- sizes (kiv/cold_store.py:111-120) --
    @property
    def cold_length(self) -> int:
        return self._n

    @property
    def num_pages(self) -> int:
        return self.cold_length // self.page_size

    @property
    def num_finalized(self) -> int:
        return self.num_pages * self.page_size

    def invalidate(self) -> None:
        self.cached_step = -1
        self.cached_union = None
        self.cached_batch = -1

    def evict_from_hot(self, k_ev: np.ndarray, v_ev: np.ndarray) -> None:
        """kiv/cold_store.py:142-184: append rows; every page that fills gets a summary."""
        self.invalidate()
        before = self.num_pages
        n = k_ev.shape[2]
        self._grow(self._n + n)
        self._k[:, :, self._n:self._n + n] = to_storage(k_ev, self.storage)
        self._v[:, :, self._n:self._n + n] = to_storage(v_ev, self.storage)
        self._n += n
        S = self.page_size
        done = self.num_pages
        if done > before:
            B, H, D = self.batch, self.num_kv_heads, self.head_dim
            pages = self._k[:, :, before * S:done * S].reshape(B, H, done - before, S, D)
            self._s[:, :, before:done] = page_summary(pages, self.storage)

    # -- coarse stage (kiv/cold_store.py:203-230) --
    def coarse(self, query: np.ndarray, scaling: float, top_pages: int):
        B, Hq, Q, D = query.shape
        Np = self.num_pages
        q = to_storage(query, self.storage).astype(self.compute)
        summ = self.summaries.astype(self.compute)                      # [B, Hkv, Np, D]
        G = Hq // self.num_kv_heads
        rows = _group_rows(q, self.num_kv_heads)                        # [B, Hkv, GQ, D]
        sc = np.matmul(rows, summ.transpose(0, 1, 3, 2)) * self.compute(scaling)  # [B, Hkv, GQ, Np]
        sc = sc.reshape(B, self.num_kv_heads, G, Q, Np).reshape(B, Hq, Q, Np)
        k = min(top_pages, Np)
        top = np.zeros((B, Hq, Q, k), np.int64)
        for b in range(B):
            for h in range(Hq):
                for t in range(Q):
                    top[b, h, t] = topk_total_order(sc[b, h, t], k)
        union = np.unique(top.reshape(-1))                              # sorted (:224)
        return union, top, sc

    def candidates(self, union: np.ndarray) -> np.ndarray:
        """kiv/cold_store.py:227-230 and :252-262: token ids of the union pages, then the partial page."""
        S = self.page_size
        fin = (union[:, None] * S + np.arange(S)[None, :]).reshape(-1)
        part = np.arange(self.num_finalized, self.cold_length)
        return np.concatenate([fin, part]).astype(np.int64)

    def fine(self, query: np.ndarray, scaling: float, cand_idx: np.ndarray, top_p: int):
        """kiv/cold_store.py:301, :332-347: fine scores, max over heads/positions, top-P."""
        B, Hq, Q, D = query.shape
        q = to_storage(query, self.storage).astype(self.compute)
        kc = self._k[:, :, cand_idx, :].astype(self.compute, copy=False)  # [B, Hkv, C, D]
        rows = _group_rows(q, self.num_kv_heads)
        sc = np.matmul(rows, kc.transpose(0, 1, 3, 2)) * self.compute(scaling)  # [B, Hkv, GQ, C]
        agg = sc.max(axis=(1, 2)).astype(np.float64)                    # [B, C]
        P = min(top_p, self.cold_length, cand_idx.shape[0])
        sel = np.zeros((B, P), np.int64)
        for b in range(B):
            pos = topk_total_order(agg[b], P)
            sel[b] = np.sort(cand_idx[pos])
        return agg, sel

    def gather(self, sel: np.ndarray):
        """kiv/cold_store.py:358-362: K and V rows of the selected tokens, per batch row."""
        B = sel.shape[0]
        k = np.stack([self._k[b][:, sel[b], :] for b in range(B)])
        v = np.stack([self._v[b][:, sel[b], :] for b in range(B)])
        return k, v

    def retrieve_top_kv(self, query: np.ndarray, scaling: float, top_pages: int,
                        top_p: int, step: int = -1) -> RetrievalResult | None:
        """kiv/cold_store.py:283-371, including the shared-layer reuse keyed by ``step``."""
        if self.cold_length == 0:
            return None
        B = query.shape[0]
        coarse_scores = None
        top = None
        skipped = False
        if step >= 0 and step == self.cached_step and self.cached_union is not None \
                and self.cached_batch == B:
            union = self.cached_union
            skipped = True
        else:
            if self.num_pages > 0:
                union, top, coarse_scores = self.coarse(query, scaling, top_pages)
            else:
                union = np.zeros((0,), np.int64)
                skipped = True
            self.cached_union = union
            self.cached_batch = B
            if step >= 0:
                self.cached_step = step
        cand = self.candidates(union)
        agg, sel = self.fine(query, scaling, cand, top_p)
        k_out, v_out = self.gather(sel)
        return RetrievalResult(union, top, coarse_scores, cand, agg, sel, k_out, v_out, skipped)


# --------------------------------------------------------------------------
# attention (kiv/middleware.py:330-352 + HF eager_attention_forward)
# --------------------------------------------------------------------------

def causal_hot_mask(batch: int, q_len: int, hot_len: int) -> np.ndarray:
    """Additive mask [B, 1, Q, hot] for Q new tokens that are the last Q hot rows."""
    i = np.arange(q_len)[:, None]
    j = np.arange(hot_len)[None, :]
    m = np.where(j <= hot_len - q_len + i, 0.0, -np.inf)
    return np.broadcast_to(m, (batch, 1, q_len, hot_len)).astype(np.float64)


def eager_attention(query, k_cold, v_cold, k_hot, v_hot, scaling, hot_mask=None,
                    softcap=None):
    """Attention over ``[cold ; hot]`` keys with all cold columns attendable.

    ``query`` [B, Hq, Q, D]; keys/values [B, Hkv, *, D]; ``hot_mask`` additive
    [B, 1|Hq, Q, hot] or None.  Returns [B, Q, Hq, D] float64 (the layout the HF
    attention interface returns).  Softmax in float64.
    """
    q = np.asarray(query, np.float64)
    B, Hq, Q, D = q.shape
    parts_k = [x for x in (k_cold, k_hot) if x is not None and x.shape[2] > 0]
    parts_v = [x for x in (v_cold, v_hot) if x is not None and x.shape[2] > 0]
    K = np.concatenate(parts_k, axis=2).astype(np.float64)
    V = np.concatenate(parts_v, axis=2).astype(np.float64)
    hkv = K.shape[1]
    G = Hq // hkv
    K = np.repeat(K, G, axis=1)
    V = np.repeat(V, G, axis=1)
    s = np.matmul(q, K.transpose(0, 1, 3, 2)) * float(scaling)
    if softcap is not None:
        s = np.tanh(s / softcap) * softcap
    n_cold = 0 if k_cold is None else k_cold.shape[2]
    if hot_mask is not None:
        s[..., n_cold:] += np.asarray(hot_mask, np.float64)
    m = s.max(axis=-1, keepdims=True)
    p = np.exp(s - m)
    p /= p.sum(axis=-1, keepdims=True)
    o = np.matmul(p, V)
    return o.transpose(0, 2, 1, 3)


# --------------------------------------------------------------------------
# tiered cache flow for one layer (kiv/tiered_cache.py:51-142)
# --------------------------------------------------------------------------

@dataclass
class OracleLayer:
    """One independent KV layer: hot window plus its cold store."""

    store: OracleStore
    hot_budget: int
    hot_k: np.ndarray = field(init=False)
    hot_v: np.ndarray = field(init=False)
    prefill_complete: bool = field(default=False, init=False)

    def __post_init__(self):
        s = self.store
        shape = (s.batch, s.num_kv_heads, 0, s.head_dim)
        self.hot_k = np.zeros(shape, np.float32)
        self.hot_v = np.zeros(shape, np.float32)

    def _evict(self, n: int) -> None:
        self.store.evict_from_hot(self.hot_k[:, :, :n], self.hot_v[:, :, :n])
        self.hot_k = self.hot_k[:, :, n:]
        self.hot_v = self.hot_v[:, :, n:]

    def update(self, k: np.ndarray, v: np.ndarray) -> None:
        """tiered_cache.py:107-142: append, then (after prefill) evict above budget."""
        st = self.store.storage
        self.hot_k = np.concatenate([self.hot_k, to_storage(k, st)], axis=2)
        self.hot_v = np.concatenate([self.hot_v, to_storage(v, st)], axis=2)
        if self.prefill_complete and self.hot_k.shape[2] > self.hot_budget:
            self._evict(self.hot_k.shape[2] - self.hot_budget)

    def evict_to_cap(self, cap: int) -> None:
        """tiered_cache.py:74-85."""
        if self.hot_k.shape[2] > cap:
            self._evict(self.hot_k.shape[2] - cap)

    def mark_prefill_complete(self) -> None:
        """tiered_cache.py:51-53, 87-105."""
        self.prefill_complete = True
        self.evict_to_cap(self.hot_budget)


def decode_step(layer: OracleLayer, query, step_k, step_v, scaling, top_pages, top_p,
                step=-1, hot_mask=None, softcap=None):
    """One layer-step: update (with eviction), retrieval, attention over [cold ; hot]."""
    layer.update(step_k, step_v)
    res = layer.store.retrieve_top_kv(query, scaling, top_pages, top_p, step)
    q = to_storage(query, layer.store.storage)
    if res is None:
        out = eager_attention(q, None, None, layer.hot_k, layer.hot_v, scaling, hot_mask, softcap)
    else:
        out = eager_attention(q, res.k_out, res.v_out, layer.hot_k, layer.hot_v, scaling,
                              hot_mask, softcap)
    return res, out


# --------------------------------------------------------------------------
# parity helpers
# --------------------------------------------------------------------------

def topk_set_mismatch(got: np.ndarray, want: np.ndarray, score_of, k: int,
                      all_scores: np.ndarray, rtol: float = 1e-6) -> list:
    """Elements in the symmetric difference of two top-k sets whose score is NOT
    within ``rtol`` (relative) of the k-th largest score.  Empty list == parity."""
    got = set(int(x) for x in np.asarray(got).reshape(-1))
    want = set(int(x) for x in np.asarray(want).reshape(-1))
    if len(got) != len(want):
        return [("size", len(got), len(want))]
    diff = got ^ want
    if not diff:
        return []
    srt = np.sort(np.asarray(all_scores, np.float64).reshape(-1))[::-1]
    boundary = srt[min(k, srt.shape[0]) - 1]
    band = rtol * max(abs(boundary), 1e-30)
    return [(i, score_of(i), boundary) for i in sorted(diff)
            if abs(score_of(i) - boundary) > band]
