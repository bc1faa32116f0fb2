"""HBM-resident cold store with page-based coarse-to-fine retrieval.

Drop-in for the reference's ``ColdKVStore`` (kiv/cold_store.py:35-414): same
constructor, ``evict_from_hot``, ``retrieve_top_kv``, ``cold_length``,
``num_pages``, ``reset``, ``telemetry_snapshot``, ``reset_telemetry``,
``memory_bytes`` and the ``_cached_*`` attributes outside code clears.

What differs is where the data lives and who computes:

* cold K/V are preallocated token slots in HBM (``[B, Hkv, capacity, D]``);
  page summaries are written by the eviction kernel in the same pass that
  copies the rows -- nothing is re-concatenated and nothing goes to host memory;
* the hot window of the owning layer lives here too, as a buffer whose start
  and length are kept in device memory next to the cold length, so the decode
  step launches the same kernels with the same arguments every time;
* every step of the retrieval runs in ``libkiv_b200.so`` (C ABI, ``include/
  kiv_b200.h``), called through its PyTorch operators ``torch.ops.kiv.*``
  (``kiv_b200.ops``); there is no CPU or PyTorch fallback, a missing library
  raises.

The store can be one shard of a cold tier partitioned over GPUs (page p on
shard p % shard_count); the collective steps then go through ``comm``.
"""

from __future__ import annotations

import ctypes
import weakref
import math
import os

import torch

from . import _native as nat
from . import ops
from .config import KIVConfig
from .model_topology import ModelTopology
from .telemetry import RetrievalTelemetry

_MIN_COLD = 8192


def _free_host(ptr: int) -> None:
    try:
        nat.lib().kiv_host_free(ptr)
    except Exception:  # pragma: no cover - interpreter shutdown
        pass


class ColdKVStore:
    """Cold tier (and hot window buffer) of one independent KV layer."""

    def __init__(self, kiv_config: KIVConfig, topology: ModelTopology, device: torch.device,
                 *, shard_rank: int = 0, shard_count: int = 1, comm=None, batch_comm=None) -> None:
        self.kiv_config = kiv_config
        self.device = torch.device(device)
        self._num_kv_groups = topology.num_query_heads // topology.num_kv_heads
        self._num_kv_heads = topology.num_kv_heads
        self._num_query_heads = topology.num_query_heads
        self._head_dim = topology.head_dim
        self._page_size = kiv_config.page_size
        self._shard_rank = shard_rank
        self._shard_count = shard_count
        self._comm = comm
        # sequence sharding: this store holds the calling rank's sequences;
        # the page union is OR-reduced over batch_comm's ranks
        self._batch_comm = batch_comm
        if shard_count > 1 and batch_comm is not None:
            raise ValueError("a store is either page-sharded or sequence-sharded, not both")
        if shard_count > 1 and comm is None:
            raise ValueError("a sharded ColdKVStore needs a comm")
        self._batch: int | None = None
        self._dtype: torch.dtype | None = None
        self._k = self._v = self._summ = None
        # pinned host overflow tier (kiv_host_alloc'd, freed with the store)
        self._host_k = self._host_v = None
        self._host_tokens = 0
        self._page_sums: torch.Tensor | None = None
        self._hk = self._hv = None
        self._hot_cap = 0
        self._state: torch.Tensor | None = None
        # host mirrors of the device state (advanced by the same rules)
        self._cold_len = 0
        self._hot_start = 0
        self._hot_len = 0
        self._desc: nat.StoreDesc | None = None
        self._op_tensors: list | None = None
        self._ws: dict[tuple, tuple] = {}
        self._bufs: dict[tuple, torch.Tensor] = {}
        self._fx_ok: dict[tuple, bool] = {}
        self._fine_x = False      # the last sharded fine pass was the candidate exchange
        # shared-layer candidate reuse (attribute names of the reference)
        self._cached_candidate_k: torch.Tensor | None = None
        self._cached_candidate_v: torch.Tensor | None = None
        self._cached_candidate_idx: torch.Tensor | None = None
        self._cached_step: int = -1
        self._cached_ws_key: tuple | None = None
        self._telemetry = RetrievalTelemetry(kiv_config.telemetry)
        # optional event recorder (``record(name)``) used by the benchmark to time
        # the fine scoring kernel on its own stream
        self._profile = None

    # ------------------------------------------------------------------ sizes
    @property
    def cold_length(self) -> int:
        return self._cold_len

    @property
    def num_pages(self) -> int:
        return self._cold_len // self._page_size

    @property
    def _num_finalized(self) -> int:
        return self.num_pages * self._page_size

    @property
    def _partial_len(self) -> int:
        return self._cold_len % self._page_size

    @property
    def hot_length(self) -> int:
        return self._hot_len

    @property
    def initialized(self) -> bool:
        return self._state is not None

    def _local_pages(self, n_global_pages: int) -> int:
        r, n = self._shard_rank, self._shard_count
        return (n_global_pages - r + n - 1) // n if n_global_pages > r else 0

    # ------------------------------------------------------------ allocation
    def _ensure_alloc(self, batch: int, dtype: torch.dtype) -> None:
        if self._state is not None:
            if batch != self._batch:
                raise ValueError(f"store holds batch {self._batch}, got {batch}")
            return
        if self.device.type != "cuda":
            raise nat.KIVNativeError(
                f"ColdKVStore runs on CUDA devices only (got {self.device}); the B200 kernels "
                "are the only implementation")
        nat.dtype_code(dtype)
        ops.load()
        self._batch, self._dtype = batch, dtype
        self._state = torch.zeros(nat.STATE_WORDS, dtype=torch.int64, device=self.device)
        cap = self.kiv_config.cold_capacity or _MIN_COLD
        if self.kiv_config.host_tokens > 0:
            self._alloc_tiered(self._round_local(cap), self._round_local(self.kiv_config.host_tokens))
        else:
            self._alloc_cold(self._round_local(cap))

    def _round_local(self, global_tokens: int) -> int:
        """Local token slots that hold the pages of ``global_tokens`` cold tokens
        -- the same on every shard (the largest shard's page count), so the
        shards' stores, workspaces and exchange arenas have one layout."""
        pages = math.ceil(global_tokens / self._page_size)
        return max(1, -(-pages // self._shard_count)) * self._page_size

    @property
    def replicated_summaries(self) -> bool:
        """Page-sharded stores keep every global page's summary on every shard:
        the coarse pass is then exact on each shard with no exchange."""
        return self._shard_count > 1 and self.kiv_config.host_tokens == 0

    def _alloc_cold(self, cap: int) -> None:
        B, H, D, S = self._batch, self._num_kv_heads, self._head_dim, self._page_size
        k = torch.empty(B, H, cap, D, dtype=self._dtype, device=self.device)
        v = torch.empty_like(k)
        # summaries: this shard's pages, or every global page the shards hold
        # (their local page counts differ by at most one)
        n_summ = (cap // S + 1) * self._shard_count if self.replicated_summaries else cap // S
        s = torch.empty(B, H, n_summ, D, dtype=self._dtype, device=self.device)
        if self.replicated_summaries and self._page_sums is None:
            # running fp32 sums of the page being filled (two slots: read one, write the other)
            self._page_sums = torch.zeros(2, B, H, D, dtype=torch.float32, device=self.device)
        if self._k is not None:
            old = self._k.shape[2]
            k[:, :, :old].copy_(self._k)
            v[:, :, :old].copy_(self._v)
            s[:, :, :self._summ.shape[2]].copy_(self._summ)
        self._k, self._v, self._summ = k, v, s
        self._desc = None
        self._op_tensors = None
        self._ws.clear()
        self._cached_ws_key = None

    def _alloc_tiered(self, ring: int, host: int) -> None:
        """HBM ring of `ring` local token slots plus the staging pages, summaries
        for ring + host pages, and the pinned host tier of `host` slots."""
        B, H, D, S = self._batch, self._num_kv_heads, self._head_dim, self._page_size
        stage = self.kiv_config.stage_pages
        if ring // S < 2:
            raise ValueError("the HBM ring of a tiered store needs at least 2 pages")
        self._k = torch.empty(B, H, ring + stage * S, D, dtype=self._dtype, device=self.device)
        self._v = torch.empty_like(self._k)
        self._summ = torch.empty(B, H, (ring + host) // S, D, dtype=self._dtype, device=self.device)
        self._ring_pages = ring // S
        self._host_tokens = host
        self._host_k = self._host_tensor(B, H, host, D)
        self._host_v = self._host_tensor(B, H, host, D)
        self._desc = None
        self._op_tensors = None
        self._ws.clear()
        self._cached_ws_key = None

    def _host_tensor(self, B: int, H: int, n: int, D: int) -> torch.Tensor:
        """A [B, H, n, D] CPU tensor over pinned, device-mapped memory."""
        esz = torch.empty((), dtype=self._dtype).element_size()
        nbytes = B * H * n * D * esz
        ptr = ctypes.c_void_p()
        nat.check(nat.lib().kiv_host_alloc(nbytes, ctypes.byref(ptr)), "host_alloc")
        weakref.finalize(self, _free_host, ptr.value)
        buf = (ctypes.c_char * nbytes).from_address(ptr.value)
        return torch.frombuffer(buf, dtype=torch.uint8).view(self._dtype).view(B, H, n, D)

    @property
    def tiered(self) -> bool:
        """True when the store has a pinned host overflow tier."""
        return self._host_tokens > 0

    def _evict_limit(self) -> int | None:
        """Most cold rows one eviction call may move with a host tier (each
        call may reach at most the ring's pages), None without one."""
        if not self.tiered:
            return None
        return max(1, (self._ring_pages - 2) * self._page_size)

    def reserve(self, cold_tokens: int, hot_rows: int | None = None) -> None:
        """Preallocate room for ``cold_tokens`` cold tokens (and a hot buffer of
        ``hot_rows``) so later steps never reallocate (CUDA-graph capture)."""
        if self._state is None:
            raise RuntimeError("reserve() needs an initialized store (evict or append first)")
        need = self._round_local(cold_tokens)
        if self.tiered:
            if need > self._ring_pages * self._page_size + self._host_tokens:
                raise nat.KIVNativeError(f"{cold_tokens} cold tokens exceed the HBM ring + host tier")
        elif need > self._k.shape[2]:
            self._alloc_cold(need)
        if hot_rows is not None and hot_rows > self._hot_cap:
            self._grow_hot(hot_rows)

    def _ensure_cold_room(self, new_cold_len: int) -> None:
        need = self._round_local(new_cold_len)
        if self.tiered:
            if need > self._ring_pages * self._page_size + self._host_tokens:
                raise nat.KIVNativeError(
                    f"cold tier full: {new_cold_len} tokens exceed the HBM ring "
                    f"({self._ring_pages * self._page_size}) + host tier ({self._host_tokens}) slots")
            return
        cap = self._k.shape[2]
        if need > cap:
            self._alloc_cold(max(need, self._round_local(2 * self._cold_len)))

    def _grow_hot(self, cap: int) -> None:
        B, H, D = self._batch, self._num_kv_heads, self._head_dim
        hk = torch.empty(B, H, cap, D, dtype=self._dtype, device=self.device)
        hv = torch.empty_like(hk)
        if self._hk is not None and self._hot_len > 0:
            a, n = self._hot_start, self._hot_len
            hk[:, :, :n].copy_(self._hk[:, :, a:a + n])
            hv[:, :, :n].copy_(self._hv[:, :, a:a + n])
        self._hk, self._hv, self._hot_cap = hk, hv, cap
        self._set_hot_start(0)
        self._desc = None
        self._op_tensors = None
        self._ws.clear()
        self._cached_ws_key = None

    def _set_hot_start(self, start: int) -> None:
        self._hot_start = start
        self._state[nat.ST_HOT_START].fill_(start)

    def _ensure_hot_room(self, n_new: int) -> None:
        """Keep start + len + n_new within the buffer (grow or compact)."""
        need = self._hot_len + n_new
        if need > self._hot_cap:
            self._grow_hot(need + max(self.kiv_config.hot_slack, n_new) + self.kiv_config.hot_budget)
        elif self._hot_start + need > self._hot_cap:
            a, n = self._hot_start, self._hot_len
            if n > 0:
                if a >= n:
                    self._hk[:, :, :n].copy_(self._hk[:, :, a:a + n])
                    self._hv[:, :, :n].copy_(self._hv[:, :, a:a + n])
                else:
                    self._hk[:, :, :n].copy_(self._hk[:, :, a:a + n].clone())
                    self._hv[:, :, :n].copy_(self._hv[:, :, a:a + n].clone())
            self._set_hot_start(0)

    def descriptor(self) -> nat.StoreDesc:
        if self._desc is None:
            self._desc = nat.StoreDesc(
                self._batch, self._num_kv_heads, self._head_dim, self._page_size,
                nat.dtype_code(self._dtype), self._shard_rank, self._shard_count, 0,
                self._k.shape[2], self._hot_cap,
                self._k.data_ptr(), self._v.data_ptr(), self._summ.data_ptr(),
                nat.ptr(self._hk), nat.ptr(self._hv), self._state.data_ptr(),
                self._host_tokens, nat.ptr(self._host_k), nat.ptr(self._host_v),
                self.kiv_config.stage_pages if self.tiered else 0, self._store_flags(), nat.ptr(self._page_sums))
        return self._desc

    def _store_flags(self) -> int:
        return nat.STORE_REPL_SUMMARIES if self.replicated_summaries else 0

    def _op_store(self, hot_hint: int = 0):
        """The store as the operators take it: (8 tensors, 5 ints)."""
        if self._op_tensors is None:
            empty = self._empty()
            self._op_tensors = [self._k, self._v, self._summ,
                                self._hk if self._hk is not None else empty,
                                self._hv if self._hv is not None else empty, self._state,
                                self._host_k if self._host_k is not None else empty,
                                self._host_v if self._host_v is not None else empty,
                                self._page_sums if self._page_sums is not None else empty]
        geom = [self._page_size, self._shard_rank, self._shard_count, int(hot_hint),
                self.kiv_config.stage_pages if self.tiered else 0, self._store_flags()]
        return self._op_tensors, geom

    def _empty(self) -> torch.Tensor:
        return torch.empty(0, dtype=self._dtype, device=self.device)

    def _rows(self, x: torch.Tensor) -> torch.Tensor:
        """New K/V rows as the kernels want them: store dtype/device, 16-byte aligned rows."""
        if x.device != self.device or x.dtype != self._dtype:
            x = x.to(device=self.device, dtype=self._dtype)
        eb = x.element_size()
        if (x.stride(-1) != 1 or x.data_ptr() % 16 or any((s * eb) % 16 for s in x.stride()[:3])):
            x = x.contiguous()
        return x

    # ------------------------------------------------------------- eviction
    def _invalidate_candidates(self) -> None:
        self._cached_candidate_k = None
        self._cached_candidate_v = None
        self._cached_candidate_idx = None
        self._cached_step = -1

    def evict_from_hot(self, k_evicted: torch.Tensor, v_evicted: torch.Tensor) -> None:
        """Append rows to the cold tier, building page summaries as pages fill
        (kiv/cold_store.py:142-184).  The hot window is not touched."""
        self._invalidate_candidates()
        B, _, n, _ = k_evicted.shape
        self._ensure_alloc(B, k_evicted.dtype)
        if n == 0:
            return
        limit = self._evict_limit()
        if limit is not None and n > limit:
            for a in range(0, n, limit):
                self.evict_from_hot(k_evicted[:, :, a:a + limit], v_evicted[:, :, a:a + limit])
            return
        k, v = self._rows(k_evicted), self._rows(v_evicted)
        if any(m > 1 and a != b for m, a, b in zip(k.shape, k.stride(), v.stride())):
            k, v = k.contiguous(), v.contiguous()
        self._ensure_cold_room(self._cold_len + n)
        with torch.cuda.device(self.device):
            ops.call(ops.kiv().append_evict, *self._op_store(), k, v, nat.KEEP_DIRECT, n)
        self._cold_len += n

    def append_and_evict(self, k_new: torch.Tensor | None, v_new: torch.Tensor | None,
                         keep: int) -> int:
        """Append new rows to the hot window, then move the oldest
        ``max(0, hot + new - keep)`` rows to the cold tier (``keep < 0``: none).
        One kernel launch.  Returns the number of rows evicted."""
        if k_new is not None:
            B, n = k_new.shape[0], k_new.shape[2]
            self._ensure_alloc(B, k_new.dtype)
        else:
            n = 0
            if self._state is None:
                return 0
        n_ev = 0 if keep < 0 else min(max(self._hot_len + n - keep, 0), self._hot_len + n)
        if n == 0 and n_ev == 0:
            return 0
        limit = self._evict_limit()
        if limit is not None and n_ev > limit:
            # a host tier bounds the pages one call reaches: append, then evict in steps
            if n > 0:
                self.append_and_evict(k_new, v_new, -1)
            done = 0
            while done < n_ev:
                c = min(limit, n_ev - done)
                self.append_and_evict(None, None, self._hot_len - c)
                done += c
            return n_ev
        self._ensure_hot_room(n)
        self._ensure_cold_room(self._cold_len + n_ev)
        k = v = None
        if n > 0:
            k, v = self._rows(k_new), self._rows(v_new)
            if any(n > 1 and a != b for n, a, b in zip(k.shape, k.stride(), v.stride())):
                k, v = k.contiguous(), v.contiguous()
        with torch.cuda.device(self.device):
            ops.call(ops.kiv().append_evict, *self._op_store(), k, v, keep, n_ev)
        self._cold_len += n_ev
        self._hot_start += n_ev
        self._hot_len += n - n_ev
        if n_ev > 0:
            self._invalidate_candidates()
        return n_ev

    # ---------------------------------------------------------- hot window
    def hot_keys(self) -> torch.Tensor:
        a, n = self._hot_start, self._hot_len
        return self._hk[:, :, a:a + n]

    def hot_values(self) -> torch.Tensor:
        a, n = self._hot_start, self._hot_len
        return self._hv[:, :, a:a + n]

    def set_hot(self, keys: torch.Tensor, values: torch.Tensor) -> None:
        """Replace the hot window content (HF layer assignment, crop, reorder)."""
        B, _, n, _ = keys.shape
        self._ensure_alloc(B, keys.dtype)
        if self._hk is not None:
            base = self._hk.untyped_storage().data_ptr(), self._hv.untyped_storage().data_ptr()
            if keys.untyped_storage().data_ptr() in base or values.untyped_storage().data_ptr() in base:
                keys, values = keys.clone(), values.clone()
        if n > self._hot_cap:
            self._hot_len = 0
            self._grow_hot(n + self.kiv_config.hot_slack + self.kiv_config.hot_budget)
        self._hk[:, :, :n].copy_(keys)
        self._hv[:, :, :n].copy_(values)
        self._hot_len = n
        self._set_hot_start(0)
        self._state[nat.ST_HOT_LEN].fill_(n)

    def truncate_hot(self, n: int) -> None:
        self._hot_len = n
        self._state[nat.ST_HOT_LEN].fill_(n)

    # ------------------------------------------------------------ retrieval
    def _query(self, query: torch.Tensor) -> torch.Tensor:
        if query.device != self.device or query.dtype != self._dtype:
            query = query.to(device=self.device, dtype=self._dtype)
        eb = query.element_size()
        if (query.stride(-1) != 1 or query.data_ptr() % 16
                or any((s * eb) % 16 for s in query.stride()[:3])):
            query = query.contiguous()
        return query

    def _workspace(self, qa: tuple, B: int, Hq: int, Q: int, top_pages: int, top_p: int):
        """(key, (workspace tensor, layout words)) for this query shape."""
        key = (B, Hq, Q, top_pages, top_p)
        ws = self._ws.get(key)
        if ws is None:
            lay = ops.call(ops.kiv().workspace_layout, *self._op_store(), qa[0], top_pages, top_p)
            nbytes = lay[10]
            if nbytes == 0:
                raise nat.KIVNativeError("workspace size: the store/query shape was rejected")
            # zeroed once: the page-flag array must start clear (kernels keep it clear)
            buf = torch.zeros(nbytes + 256, dtype=torch.uint8, device=self.device)
            off = (-buf.data_ptr()) % 256
            buf = buf[off:off + nbytes]
            ws = (buf, tuple(lay[:10]))
            self._ws[key] = ws
        return key, ws

    def _buffer(self, name: str, shape: tuple, dtype: torch.dtype) -> torch.Tensor:
        key = (name,) + tuple(shape) + (dtype,)
        t = self._bufs.get(key)
        if t is None:
            t = torch.empty(shape, dtype=dtype, device=self.device)
            self._bufs[key] = t
        return t

    def _expected_P(self, top_pages: int, top_p: int) -> int | None:
        """Selected count when it follows from host-known sizes, else None."""
        p = min(top_p, self._cold_len)
        guaranteed = min(top_pages, self.num_pages) * self._page_size + self._partial_len
        return p if p <= guaranteed else None

    def _select(self, query: torch.Tensor, scaling: float, kiv_config: KIVConfig, step: int,
                softcap: float | None = None, global_sel: bool = True):
        """Coarse (or reuse) + fine.  Returns (sel [B, top_p] int32, ws key, ws, qdesc)."""
        B, Hq, Q, _ = query.shape
        top_pages, top_p = kiv_config.top_pages, kiv_config.top_p
        qa = (query, float(scaling), int(top_pages), int(top_p), float(softcap or 0.0))
        wkey, (ws, lay) = self._workspace(qa, B, Hq, Q, top_pages, top_p)
        K = ops.kiv()
        so = self._op_store()
        reuse = (step >= 0 and step == self._cached_step and self._cached_candidate_k is not None
                 and self._cached_candidate_k.shape[0] == B and self._cached_ws_key == wkey)
        if reuse:
            self._telemetry.record_coarse_skipped(cold_length=self._cold_len)
        else:
            if self._profile is not None:
                self._profile.record("coarse_begin")
            if self._shard_count == 1:
                ops.call(K.coarse_select, *so, *qa, ws, None, None)
                if self._batch_comm is not None and self._batch_comm.size > 1:
                    # the union spans the whole batch, held by all ranks
                    words = (lay[7] + 31) // 32
                    self._batch_comm.all_or_bits(ws[lay[1]:lay[1] + 4 * words].view(torch.int32))
            else:
                self._sharded_coarse(qa, ws, B * Hq * Q, top_pages)
            marker = self._buffer("marker", (B, 0), torch.int8)
            self._cached_candidate_k = marker
            self._cached_candidate_v = marker
            self._cached_candidate_idx = ws[lay[2]:lay[2] + 4 * lay[8]].view(torch.int32)
            self._cached_ws_key = wkey
            if step >= 0:
                self._cached_step = step
        sel = self._buffer("sel", (B, top_p), torch.int32)
        if self._shard_count == 1:
            prof = self._profile
            if prof is not None:
                prof.record("fine_score_begin")
            ops.call(K.fine_score, *so, *qa, ws)
            if prof is not None:
                prof.record("fine_score_end")
            ops.call(K.fine_topk, *so, *qa, ws, sel, None)
            if prof is not None:
                prof.record("fine_topk_end")
            sel_local = sel
        else:
            sel_local = self._sharded_fine(qa, ws, B, top_p, sel if global_sel else None)
        if not reuse:
            # the fine scorer materializes the page union the coarse pass marked
            if self.num_pages > 0:
                uni = ws[lay[2]:lay[2] + 4 * lay[8]].view(torch.int32)
                self._telemetry.record_coarse(state=self._state, union=uni, num_pages=self.num_pages,
                                              cold_length=self._cold_len,
                                              n_scores=B * Hq * Q * self._local_pages(self.num_pages))
            else:
                self._telemetry.record_coarse_skipped(cold_length=self._cold_len)
        return sel, sel_local, ws, qa

    def _record_fine(self, sel: torch.Tensor, P: int | None, top_p: int) -> None:
        if self._telemetry.enabled:
            if P is None:
                P = self.read_state()[nat.ST_SEL]
            self._telemetry.record_fine(state=self._state, selected=sel, actual_P=int(P),
                                        requested_P=top_p, cold_length=self._cold_len,
                                        n_scores=0)

    def retrieve_indices(self, query: torch.Tensor, scaling: float, kiv_config: KIVConfig,
                         step: int = -1) -> tuple[torch.Tensor, int] | None:
        """Global token ids selected for each batch row: ``(sel [B, top_p], P)``;
        the first P entries of each row are valid, ascending."""
        if self._cold_len == 0:
            return None
        query = self._query(query)
        with torch.cuda.device(self.device):
            sel, _, _, _ = self._select(query, scaling, kiv_config, step)
            P = self._expected_P(kiv_config.top_pages, kiv_config.top_p)
            if P is None:
                P = int(self.read_state()[nat.ST_SEL])
            self._record_fine(sel, P, kiv_config.top_p)
        return sel, P

    def retrieve_top_kv(self, query: torch.Tensor, scaling: float, kiv_config: KIVConfig,
                        step: int = -1) -> tuple[torch.Tensor, torch.Tensor] | tuple[None, None]:
        """Coarse-to-fine retrieval returning the selected K and V, ``[B, Hkv, P, D]``
        each, or ``(None, None)`` when the cold tier is empty (kiv/cold_store.py:283-371).
        Rows come in ascending token order (the reference returns them in
        descending-score order; attention over them does not depend on it)."""
        r = self.retrieve_indices(query, scaling, kiv_config, step)
        if r is None:
            return None, None
        sel, P = r
        B = sel.shape[0]
        out_k = torch.empty(B, self._num_kv_heads, P, self._head_dim, dtype=self._dtype,
                            device=self.device)
        out_v = torch.empty_like(out_k)
        if self._shard_count > 1:
            out_k.zero_()
            out_v.zero_()
        with torch.cuda.device(self.device):
            ops.call(ops.kiv().gather_rows, *self._op_store(), sel, P, out_k, out_v)
        if self._shard_count > 1:
            self._comm.all_reduce_sum(out_k)
            self._comm.all_reduce_sum(out_v)
        return out_k, out_v

    def attend(self, query: torch.Tensor, scaling: float, kiv_config: KIVConfig, step: int = -1,
               *, mask_add: torch.Tensor | None = None, causal: bool = False,
               softcap: float | None = None, out: torch.Tensor | None = None) -> torch.Tensor:
        """Fused retrieval attention over [selected cold ; hot window]:
        ``query [B, Hq, Q, D] -> [B, Q, Hq, D]`` (the HF attention-interface layout).

        ``mask_add``: float32 additive mask over the hot rows ``[B, 1|Hq, Q, hot]``;
        ``causal``: query position i sees hot row j iff j <= hot - Q + i.
        Cold rows are always attendable (kiv/mask_utils.py:8-38)."""
        query = self._query(query)
        B, Hq, Q, D = query.shape
        if out is None:
            out = torch.empty(B, Q, Hq, D, dtype=self._dtype, device=self.device)
        elif (out.shape != (B, Q, Hq, D) or out.dtype != self._dtype or not out.is_contiguous()
              or out.device != self.device):
            raise ValueError("out must be a contiguous [B, Q, Hq, D] tensor of the store dtype")
        if mask_add is not None and (mask_add.dtype != torch.float32 or mask_add.stride(-1) != 1):
            raise nat.KIVNativeError("mask must be float32 with a contiguous last dim")
        with torch.cuda.device(self.device):
            if self._cold_len > 0:
                sel, sel_local, ws, qa = self._select(query, scaling, kiv_config, step, softcap,
                                                      global_sel=self._telemetry.enabled)
                if self._telemetry.enabled:
                    self._record_fine(sel, self._expected_P(kiv_config.top_pages, kiv_config.top_p),
                                      kiv_config.top_p)
            else:
                qa = (query, float(scaling), int(kiv_config.top_pages), int(kiv_config.top_p),
                      float(softcap or 0.0))
                _, (ws, lay) = self._workspace(qa, B, Hq, Q, kiv_config.top_pages, kiv_config.top_p)
                sel_local = self._buffer("sel", (B, kiv_config.top_p), torch.int32)
                ws[lay[4]:lay[4] + 4 * self._batch].zero_()
            K = ops.kiv()
            so = self._op_store(hot_hint=self._hot_len)
            if self._shard_count == 1:
                ops.call(K.attend, *so, *qa, ws, sel_local, mask_add, bool(causal), 0, 1, out, None)
                if self._profile is not None:
                    self._profile.record("attend_end")
            elif self._cold_len > 0 and self._fine_x:
                # every shard reads the selected rows from their owners' cold tiers
                pk, pv = self._comm.map_peers([self._k.data_ptr(), self._v.data_ptr()], self.device)
                ops.call(K.attend_peers, *so, *qa, ws, sel_local, mask_add, bool(causal), pk, pv, out)
                if self._profile is not None:
                    self._profile.record("attend_end")
            else:
                R = B * Hq * Q
                part = self._buffer("apart", (R, D + 4), torch.float32)
                ops.call(K.attend, *so, *qa, ws, sel_local, mask_add, bool(causal), self._shard_rank,
                         self._shard_count, None, part)
                x = self._exchange(qa)
                if x is not None:
                    ops.call(K.attend_exchange_merge, *so, *qa, part, *x, out)
                else:
                    gathered = self._buffer("apart_all", (self._shard_count, R, D + 4), torch.float32)
                    self._comm.all_gather(gathered, part)
                    ops.call(K.attend_merge, *so, *qa, gathered, out)
                if self._profile is not None:
                    self._profile.record("attend_end")
        return out

    # ---------------------------------------------------------- sharded steps
    def _exchange(self, qa: tuple):
        """Peer-memory exchange arguments ``(arenas, arena_bytes, wait_cycles)`` for
        this query shape, or None when the process group's collectives are used
        (``KIV_SHARD_EXCHANGE=collective``)."""
        if os.environ.get("KIV_SHARD_EXCHANGE", "peer") == "collective":
            return None
        qd = nat.query_desc(qa[0], qa[1], qa[2], qa[3], qa[4])
        nbytes = nat.lib().kiv_exchange_bytes(ctypes.byref(self.descriptor()), ctypes.byref(qd),
                                              self._shard_count)
        if nbytes == 0:
            raise nat.KIVNativeError("kiv_exchange_bytes rejected the store/query shape")
        x = self._comm.exchange(nbytes, self.device)
        return [int(x.arena[i]) for i in range(x.world)], int(x.arena_bytes), int(x.wait_cycles)

    def _sharded_coarse(self, qa: tuple, ws, R: int, K: int) -> None:
        kv = ops.kiv()
        so = self._op_store()
        if self.replicated_summaries:
            # every shard scores every page: the exact global union, this shard's
            # pages of it marked for the fine pass, no exchange
            ops.call(kv.coarse_select, *so, *qa, ws, None, None)
            return
        sc = self._buffer("crow_s", (R, K), torch.float32)
        pg = self._buffer("crow_p", (R, K), torch.int32)
        ops.call(kv.coarse_select, *so, *qa, ws, sc, pg)
        x = self._exchange(qa)
        if x is not None:
            ops.call(kv.coarse_exchange_merge, *so, *qa, ws, sc, pg, *x)
            return
        n = self._shard_count
        all_s = self._buffer("crow_s_all", (n, R, K), torch.float32)
        all_p = self._buffer("crow_p_all", (n, R, K), torch.int32)
        self._comm.all_gather(all_s, sc)
        self._comm.all_gather(all_p, pg)
        ops.call(kv.coarse_merge, *so, *qa, ws, all_s, all_p)

    def _fine_exchange_supported(self, qa: tuple) -> bool:
        """Whether this store/query shape takes the candidate exchange (cached per shape)."""
        key = (tuple(qa[0].shape), qa[2], qa[3], int(self._k.shape[2]))
        hit = self._fx_ok.get(key)
        if hit is None:
            qd = nat.query_desc(qa[0], qa[1], qa[2], qa[3], qa[4])
            hit = bool(nat.lib().kiv_fine_exchange_supported(ctypes.byref(self.descriptor()), ctypes.byref(qd)))
            self._fx_ok[key] = hit
        return hit

    def _sharded_fine(self, qa: tuple, ws, B: int, top_p: int, sel: torch.Tensor | None) -> torch.Tensor:
        """Fine pass of a page-sharded store; fills ``sel`` (the global list) when
        given and returns the list the attention reads.  With replicated summaries
        and peer exchange: one scorer + select over every shard's candidates (the
        keys travel through the arenas), returning the global list (the attention
        then reads every shard's rows); otherwise a local pass, then the lists'
        exchange and merge, returning this shard's part of the selection."""
        kv = ops.kiv()
        so = self._op_store()
        prof = self._profile
        x = self._exchange(qa)
        self._fine_x = x is not None and self.replicated_summaries and self._fine_exchange_supported(qa)
        if self._fine_x:
            # every shard ends with the global selection; the attention reads each
            # row from its owner (attend_peers), so no local list is needed
            if sel is None:
                sel = self._buffer("sel_global_scratch", (B, top_p), torch.int32)
            if prof is not None:
                prof.record("fine_score_begin")
            ops.call(kv.fine_exchange_select, *so, *qa, ws, *x, sel, None)
            if prof is not None:
                prof.record("fine_score_end")
                prof.record("fine_topk_end")
            return sel
        sel_local = self._buffer("sel_local", (B, top_p), torch.int32)
        lt = self._buffer("fl_t", (B, top_p), torch.int32)
        ls = self._buffer("fl_s", (B, top_p), torch.float32)
        if prof is not None:
            prof.record("fine_score_begin")
        ops.call(kv.fine_score, *so, *qa, ws)
        if prof is not None:
            prof.record("fine_score_end")
        ops.call(kv.fine_topk, *so, *qa, ws, lt, ls)
        if prof is not None:
            prof.record("fine_topk_end")
        if x is not None:
            ops.call(kv.fine_exchange_merge, *so, *qa, ws, ls, lt, *x, sel, sel_local)
            return sel_local
        n = self._shard_count
        all_t = self._buffer("fl_t_all", (n, B, top_p), torch.int32)
        all_s = self._buffer("fl_s_all", (n, B, top_p), torch.float32)
        self._comm.all_gather(all_t, lt)
        self._comm.all_gather(all_s, ls)
        if sel is None:
            sel = self._buffer("sel_global_scratch", (B, top_p), torch.int32)
        ops.call(kv.fine_merge, *so, *qa, ws, all_s, all_t, sel, sel_local)
        return sel_local

    # --------------------------------------------------------------- misc API
    def read_state(self) -> list[int]:
        """Device state words (syncs the current stream); for tests and debugging."""
        with torch.cuda.device(self.device):
            return [int(x) for x in self._state.cpu().tolist()]

    def page_summaries(self) -> torch.Tensor | None:
        """Summaries of the finalized pages this shard holds: ``[B, Hkv, pages, D]``
        -- every global page with replicated summaries (page-sharded stores),
        else this shard's pages in local order."""
        if self._summ is None:
            return None
        n = self.num_pages if self.replicated_summaries else self._local_pages(self.num_pages)
        return self._summ[:, :, :n]

    def reset(self) -> None:
        """Clear all cold storage and the hot window (buffers are kept for reuse)."""
        self._cold_len = 0
        self._hot_start = 0
        self._hot_len = 0
        if self._state is not None:
            self._state.zero_()
        self._invalidate_candidates()

    def telemetry_snapshot(self) -> dict:
        return self._telemetry.snapshot()

    def reset_telemetry(self) -> None:
        self._telemetry = RetrievalTelemetry(self.kiv_config.telemetry)

    def memory_bytes(self) -> dict[str, int]:
        """Bytes by tier.  The reference's keys are kept (its host tiers are
        empty here); the HBM-resident cold K/V and reservations are added."""
        if self._state is None:
            return {"k_index_cpu": 0, "v_store_cpu": 0, "page_summaries_gpu": 0, "partial_gpu": 0,
                    "cold_k_gpu": 0, "cold_v_gpu": 0, "reserved_gpu": 0}
        e = self._k.element_size()
        row = self._batch * self._num_kv_heads * self._head_dim * e
        local_fin = self._local_pages(self.num_pages) * self._page_size
        part = self._partial_len if (self.num_pages % self._shard_count) == self._shard_rank else 0
        reserved = sum(t.numel() * t.element_size() for t in (self._k, self._v, self._summ))
        host_k = host_v = 0
        if self.tiered:
            # pages older than the HBM ring live in the pinned host tier
            started = self._local_pages(math.ceil(self._cold_len / self._page_size))
            on_host = max(0, started - self._ring_pages) * self._page_size
            host_k = host_v = on_host * row
            local_fin = max(0, local_fin - on_host)
        return {
            "k_index_cpu": host_k,
            "v_store_cpu": host_v,
            "page_summaries_gpu": (self.num_pages if self.replicated_summaries
                                   else self._local_pages(self.num_pages)) * row,
            "partial_gpu": 2 * part * row,
            "cold_k_gpu": local_fin * row,
            "cold_v_gpu": local_fin * row,
            "reserved_gpu": reserved,
        }
