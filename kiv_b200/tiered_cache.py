"""Tiered KV cache: an HF ``DynamicCache`` whose global layers evict into an HBM cold tier.

Drop-in for the reference's ``TieredKVCache`` (kiv/tiered_cache.py:17-286):
same constructor, ``update``, ``mark_prefill_complete``, ``_evict_layer``,
``_evict_to_cap``, ``_evict_excess_all_layers``, ``get_cold_store``,
``get_mask_sizes``, ``get_seq_length``, ``truncate_to``, ``reset``,
``memory_report`` and the ``_prefill_complete`` / ``_suppress_cold`` /
``_decode_step`` / ``_total_tokens`` attributes.

The hot window of each independent KV layer is kept inside that layer's
``ColdKVStore`` (a device buffer whose start/length live in device memory), so
an update is one kernel launch that appends the new rows and moves the rows
past ``hot_budget`` into the cold tier with their page summaries -- the
reference re-concatenates the whole hot window twice per step instead.
``layer.keys`` / ``layer.values`` stay ordinary tensor views of that window.
"""

from __future__ import annotations

import logging

import torch
from transformers import DynamicCache
from transformers.cache_utils import DynamicLayer

from .cold_store import ColdKVStore
from .config import KIVConfig
from .model_topology import ModelTopology

logger = logging.getLogger(__name__)


class KIVHotLayer(DynamicLayer):
    """An HF cache layer whose K/V are the hot window held by a ColdKVStore."""

    is_sliding = False

    def __init__(self, store: ColdKVStore) -> None:
        self._store = store
        self._pending_keys: torch.Tensor | None = None
        super().__init__()

    # keys / values are views of the store's hot window; assigning replaces it
    @property
    def keys(self):
        return self._store.hot_keys() if self._store.initialized else None

    @keys.setter
    def keys(self, value):
        self._pending_keys = value

    @property
    def values(self):
        return self._store.hot_values() if self._store.initialized else None

    @values.setter
    def values(self, value):
        k = self._pending_keys
        self._pending_keys = None
        if value is None or k is None:
            return
        if k.dim() != 4 or value.dim() != 4:
            return  # lazy-initialization placeholders
        if not self._store.initialized and k.shape[2] == 0:
            return
        self._store.set_hot(k, value)

    def lazy_initialization(self, key_states, value_states) -> None:
        self.dtype, self.device = key_states.dtype, key_states.device
        self.is_initialized = True

    def update(self, key_states, value_states, *args, **kwargs):
        raise RuntimeError("KIV-managed layers are updated through TieredKVCache.update")

    def get_seq_length(self) -> int:
        return self._store.hot_length if self._store.initialized else 0

    def reset(self) -> None:
        pass


class TieredKVCache(DynamicCache):
    """Hot window + HBM cold tier per independent global layer."""

    def __init__(self, config, kiv_config: KIVConfig, topology: ModelTopology,
                 device: torch.device | None = None, *, shard_group=None, batch_group=None) -> None:
        super().__init__(config=config)
        self.kiv_config = kiv_config
        self.topology = topology
        if device is None:
            device = torch.device("cuda")
        self.device = torch.device(device)
        comm, rank, count = None, 0, 1
        if shard_group is not None:
            from .sharding import ShardComm
            comm = shard_group if isinstance(shard_group, ShardComm) else ShardComm(shard_group)
            rank, count = comm.rank, comm.size
        self.shard_comm = comm
        # sequence sharding: this rank's cache holds its own sequences of the
        # batch; the page union is taken across the ranks (the reference's
        # union spans the batch, kiv/cold_store.py:224)
        bcomm = None
        if batch_group is not None:
            if shard_group is not None:
                raise ValueError("pass shard_group (pages) or batch_group (sequences), not both")
            from .sharding import ShardComm
            bcomm = batch_group if isinstance(batch_group, ShardComm) else ShardComm(batch_group)
        self.batch_comm = bcomm
        self.cold_stores: dict[int, ColdKVStore] = {}
        for li in topology.independent_kv_layers:
            self.cold_stores[li] = ColdKVStore(kiv_config, topology, self.device,
                                               shard_rank=rank, shard_count=count, comm=comm, batch_comm=bcomm)
        need = max(topology.independent_kv_layers, default=-1) + 1
        while len(self.layers) < need:
            self.layers.append(DynamicLayer())
        for li, store in self.cold_stores.items():
            self.layers[li] = KIVHotLayer(store)
        self._prefill_complete = False
        self._suppress_cold = False
        self._total_tokens: dict[int, int] = {}
        self._decode_step: int = 0

    def _kv_source_layer_idx(self, layer_idx: int) -> int:
        return self.topology.kv_sharing_map.get(layer_idx, layer_idx)

    def mark_prefill_complete(self) -> None:
        self._prefill_complete = True
        self._evict_excess_all_layers()

    def _evict_layer(self, layer_idx: int, num_evict: int) -> None:
        """Move the oldest ``num_evict`` hot rows of a layer into its cold tier."""
        store = self.cold_stores[layer_idx]
        store.append_and_evict(None, None, keep=store.hot_length - num_evict)
        self._total_tokens[layer_idx] = store.cold_length + store.hot_length

    def _initialized(self, layer_idx: int) -> bool:
        return layer_idx < len(self.layers) and self.layers[layer_idx].is_initialized

    def _evict_to_cap(self, cap: int) -> None:
        """Evict hot rows above ``cap`` in every independent layer (bounded prefill)."""
        for li in self.topology.independent_kv_layers:
            if not self._initialized(li):
                continue
            n = self.cold_stores[li].hot_length
            if n > cap:
                self._evict_layer(li, n - cap)

    def _evict_excess_all_layers(self) -> None:
        budget = self.kiv_config.hot_budget
        for li in self.topology.independent_kv_layers:
            if not self._initialized(li):
                continue
            n = self.cold_stores[li].hot_length
            if n > budget:
                self._evict_layer(li, n - budget)
                logger.debug("Layer %d: evicted %d tokens to cold (hot=%d, cold=%d)", li, n - budget,
                             budget, self.cold_stores[li].cold_length)

    def update(self, key_states: torch.Tensor, value_states: torch.Tensor, layer_idx: int,
               *args, **kwargs) -> tuple[torch.Tensor, torch.Tensor]:
        store = self.cold_stores.get(layer_idx)
        if store is None:
            return super().update(key_states, value_states, layer_idx, *args, **kwargs)
        indep = self.topology.independent_kv_layers
        if self._prefill_complete and indep and layer_idx == indep[0]:
            self._decode_step += 1
        keep = self.kiv_config.hot_budget if self._prefill_complete else -1
        store.append_and_evict(key_states, value_states, keep)
        layer = self.layers[layer_idx]
        if not layer.is_initialized:
            layer.lazy_initialization(key_states, value_states)
        self._total_tokens[layer_idx] = store.cold_length + store.hot_length
        return layer.keys, layer.values

    def get_cold_store(self, layer_idx: int) -> ColdKVStore | None:
        if layer_idx in self.cold_stores:
            return self.cold_stores[layer_idx]
        src = self.topology.kv_sharing_map.get(layer_idx)
        return self.cold_stores.get(src) if src is not None else None

    def get_mask_sizes(self, query_length: int, layer_idx: int) -> tuple[int, int]:
        store = self.get_cold_store(layer_idx)
        src = self._kv_source_layer_idx(layer_idx)
        if store is not None and src < len(self.layers) and store.cold_length > 0:
            hot = store.hot_length if self._initialized(src) else 0
            return hot + query_length, store.cold_length
        return super().get_mask_sizes(query_length, layer_idx)

    def get_seq_length(self, layer_idx: int = 0) -> int:
        """Hot + cold length, so position ids stay right."""
        if layer_idx in self._total_tokens:
            return self._total_tokens[layer_idx]
        src = self._kv_source_layer_idx(layer_idx)
        if src in self._total_tokens:
            return self._total_tokens[src]
        if src != layer_idx:
            return super().get_seq_length(src)
        return super().get_seq_length(layer_idx)

    def reset(self) -> None:
        super().reset()
        for store in self.cold_stores.values():
            store.reset()
        self._total_tokens.clear()
        self._prefill_complete = False
        self._suppress_cold = False
        self._decode_step = 0

    # ------------------------------------------------------------ persistence
    def _store_file(self, li: int) -> str:
        """File of layer li's store: one per layer, and per rank when the cold
        pages are sharded over GPUs (each rank saves and loads its own)."""
        if self.shard_comm is not None and self.shard_comm.size > 1:
            return f"layer_{li}.rank{self.shard_comm.rank}of{self.shard_comm.size}.kivstore"
        return f"layer_{li}.kivstore"

    def save(self, directory: str) -> None:
        """Write every independent layer's store (``kiv_b200.persist`` format,
        one file per layer, per rank for page-sharded caches) and the cache
        counters to `directory`."""
        import json
        import os

        from .persist import save_store

        os.makedirs(directory, exist_ok=True)
        for li, store in self.cold_stores.items():
            if store.initialized:
                save_store(store, os.path.join(directory, self._store_file(li)), meta={"layer": li})
        state = {"prefill_complete": self._prefill_complete, "decode_step": self._decode_step,
                 "total_tokens": {str(k): v for k, v in self._total_tokens.items()}}
        with open(os.path.join(directory, "cache.json"), "w") as f:
            json.dump(state, f)

    def load(self, directory: str) -> None:
        """Restore a cache written by save() into this empty cache (same
        topology); the stores may have another HBM / host tier configuration."""
        import json
        import os

        from .persist import load_store

        with open(os.path.join(directory, "cache.json")) as f:
            state = json.load(f)
        for li, store in self.cold_stores.items():
            path = os.path.join(directory, self._store_file(li))
            if not os.path.exists(path):
                continue
            load_store(store, path)
            layer = self.layers[li]
            if not layer.is_initialized:
                layer.dtype, layer.device = store._dtype, store.device
                layer.is_initialized = True
        self._prefill_complete = bool(state["prefill_complete"])
        self._decode_step = int(state["decode_step"])
        self._total_tokens = {int(k): int(v) for k, v in state["total_tokens"].items()}

    def truncate_to(self, new_len: int) -> bool:
        """Trim every global layer to ``new_len`` tokens, inside the hot window only.

        Rejected (False, cache untouched) when ``new_len`` exceeds the current
        total or would cut into the cold tier (kiv/tiered_cache.py:194-257)."""
        layers = [li for li in self.topology.independent_kv_layers if self._initialized(li)]
        for li in layers:
            st = self.cold_stores[li]
            if new_len > st.cold_length + st.hot_length or new_len < st.cold_length:
                return False
        for li in layers:
            st = self.cold_stores[li]
            target = new_len - st.cold_length
            if target < st.hot_length:
                st.truncate_hot(target)
            self._total_tokens[li] = new_len
        for st in self.cold_stores.values():
            st._cached_candidate_k = None
            st._cached_candidate_v = None
            st._cached_candidate_idx = None
            st._cached_step = -1
        self._decode_step = 0
        return True

    def memory_report(self) -> dict:
        hot = 0
        agg = {"k_index_cpu": 0, "v_store_cpu": 0, "page_summaries_gpu": 0, "partial_gpu": 0,
               "cold_k_gpu": 0, "cold_v_gpu": 0, "reserved_gpu": 0}
        for li, st in self.cold_stores.items():
            if self._initialized(li):
                k = self.layers[li].keys
                hot += 2 * k.numel() * k.element_size()
            for key, val in st.memory_bytes().items():
                agg[key] += val
        return {
            "hot_vram_bytes": hot,
            "k_index_cpu_bytes": agg["k_index_cpu"],
            "v_store_cpu_bytes": agg["v_store_cpu"],
            "page_summaries_gpu_bytes": agg["page_summaries_gpu"],
            "total_vram_bytes": hot + agg["page_summaries_gpu"] + agg["partial_gpu"]
            + agg["cold_k_gpu"] + agg["cold_v_gpu"],
            "total_cpu_bytes": agg["k_index_cpu"] + agg["v_store_cpu"],
            "cold_kv_gpu_bytes": agg["cold_k_gpu"] + agg["cold_v_gpu"],
            "reserved_gpu_bytes": agg["reserved_gpu"],
        }
