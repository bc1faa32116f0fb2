"""vLLM V1 KV connector that shadows every new K/V row into the HBM cold tier
(kiv/vllm/connector.py:55-277).

vLLM keeps its own paged KV cache as the hot tier; after each attention layer
``save_kv_layer`` receives that layer's cache tensor and the connector copies
the step's new rows into the layer's ``ColdKVStore`` (appended straight to the
cold tier by the eviction kernel, page summaries built as pages fill).  During
decode the attention hook (``attention_hook.py``) retrieves from those stores.

Same surface and semantics as the reference connector: the KIV knobs come from
``vllm_config.extra_config["kiv"]`` (``hot_budget``, ``top_p``, ``page_size``,
``top_pages``, optional ``topology``; here also ``cold_capacity``,
``host_tokens``, ``stage_pages`` and ``telemetry`` for the tier placement);
the new rows of a step are the last
``num_prefill_tokens + num_decode_tokens`` token slots of the layer's cache
tensor, for the ``[2, slots, H, D]`` and ``[2, blocks, block_size, H, D]``
layouts; the decode step counter advances in ``wait_for_save`` once the first
decode token has been seen.  Difference: the stores live in GPU memory (the
reference shadows them to host memory).
"""

from __future__ import annotations

import logging
import re
from dataclasses import dataclass
from typing import Any

import torch

from ..cold_store import ColdKVStore
from ..config import KIVConfig
from ..model_topology import ModelTopology
from .topology import detect_topology_from_vllm

logger = logging.getLogger(__name__)

_LAYER_RE = re.compile(r"layers\.(\d+)")


@dataclass
class KIVConnectorMetadata:
    """Scheduler-to-worker metadata (nothing to carry for KIV)."""


def _parse_layer_index(layer_name: str) -> int | None:
    """Layer number in a vLLM layer name such as ``model.layers.12.self_attn``."""
    m = _LAYER_RE.search(layer_name)
    return int(m.group(1)) if m else None


def _connector_base() -> type:
    """vLLM's ``KVConnectorBase_V1`` when vLLM is importable, else ``object``."""
    try:
        from vllm.distributed.kv_transfer.kv_connector.v1.base import KVConnectorBase_V1
        return KVConnectorBase_V1
    except ImportError:
        return object


def _new_rows(kv_layer: torch.Tensor, new_tokens: int):
    """(k, v) ``[1, H, n, D]`` views of the last ``new_tokens`` token slots, or None."""
    if kv_layer.ndim == 4 and kv_layer.shape[0] == 2:            # [2, slots, H, D]
        k_all, v_all = kv_layer[0], kv_layer[1]
    elif kv_layer.ndim == 5 and kv_layer.shape[0] == 2:          # [2, blocks, bs, H, D]
        _, nb, bs, H, D = kv_layer.shape
        k_all = kv_layer[0].reshape(nb * bs, H, D)
        v_all = kv_layer[1].reshape(nb * bs, H, D)
    else:
        return None
    total = k_all.shape[0]
    lo = max(0, total - new_tokens)
    return k_all[lo:total].permute(1, 0, 2).unsqueeze(0), v_all[lo:total].permute(1, 0, 2).unsqueeze(0)


class KIVConnector(_connector_base()):
    """Shadows each layer's new K/V rows into a GPU ``ColdKVStore``.

    The base class's ``__init__`` is not called (it insists on a
    ``kv_transfer_config``); the attributes its default methods read are set
    here instead, as the reference connector does."""

    def __init__(self, vllm_config: Any, role: Any, kv_cache_config: Any = None) -> None:
        self._vllm_config = vllm_config
        self._role = role
        self._kv_cache_config = kv_cache_config
        self._connector_metadata = None
        extra = getattr(vllm_config, "extra_config", None) or {}
        kiv_extra = extra.get("kiv", {}) if isinstance(extra, dict) else {}
        # the reference's four knobs, plus this build's tier placement (HBM cold
        # capacity, pinned host overflow tier) for long contexts
        self.kiv_config = KIVConfig(hot_budget=kiv_extra.get("hot_budget", 2048),
                                    top_p=kiv_extra.get("top_p", 256),
                                    page_size=kiv_extra.get("page_size", 128),
                                    top_pages=kiv_extra.get("top_pages", 32),
                                    cold_capacity=kiv_extra.get("cold_capacity"),
                                    host_tokens=kiv_extra.get("host_tokens", 0),
                                    stage_pages=kiv_extra.get("stage_pages", 1024),
                                    telemetry=kiv_extra.get("telemetry", True))
        topology_cfg = kiv_extra.get("topology")
        self.topology = (ModelTopology.manual(**topology_cfg) if topology_cfg is not None
                         else detect_topology_from_vllm(vllm_config))
        self.cold_stores: dict[int, ColdKVStore] = {}
        self._device: torch.device | None = None
        self._kv_caches: dict[str, torch.Tensor] = {}
        self._prefill_complete = False
        self._decode_step = 0
        logger.info("KIVConnector: top_p=%d page_size=%d top_pages=%d, %d independent layers",
                    self.kiv_config.top_p, self.kiv_config.page_size, self.kiv_config.top_pages,
                    len(self.topology.independent_kv_layers))

    # -- stores ---------------------------------------------------------------------------------

    def get_cold_store(self, layer_idx: int) -> ColdKVStore | None:
        """The store of ``layer_idx``, or of the layer whose KV it reuses."""
        if layer_idx in self.cold_stores:
            return self.cold_stores[layer_idx]
        source = self.topology.kv_sharing_map.get(layer_idx)
        return self.cold_stores.get(source) if source is not None else None

    def _ensure_cold_store(self, layer_idx: int) -> ColdKVStore | None:
        if layer_idx not in self.topology.independent_kv_layers:
            return None
        store = self.cold_stores.get(layer_idx)
        if store is None:
            if self._device is None:
                self._device = torch.device("cuda")
            store = self.cold_stores[layer_idx] = ColdKVStore(self.kiv_config, self.topology, self._device)
        return store

    # -- worker side ----------------------------------------------------------------------------

    def start_load_kv(self, forward_context: Any, **kwargs: Any) -> None:
        """Nothing is loaded into vLLM's cache: retrieval happens in the attention hook."""

    def wait_for_layer_load(self, layer_name: str) -> None:
        """Nothing to wait for (see ``start_load_kv``)."""

    def save_kv_layer(self, layer_name: str, kv_layer: torch.Tensor, attn_metadata: Any,
                      **kwargs: Any) -> None:
        """Copy this step's new rows of a global layer into its cold store.

        ``layer_name`` like ``model.layers.12.self_attn``; ``kv_layer`` the
        layer's vLLM cache tensor; ``attn_metadata`` carries
        ``num_prefill_tokens`` / ``num_decode_tokens``."""
        layer_idx = _parse_layer_index(layer_name)
        if layer_idx is None or layer_idx not in self.topology.global_layer_indices:
            return
        store = self._ensure_cold_store(layer_idx)
        if store is None:
            return
        if not self._prefill_complete and getattr(attn_metadata, "num_decode_tokens", 0) > 0:
            self._prefill_complete = True
        self._shadow_kv_to_cold(layer_idx, kv_layer, attn_metadata, store)

    def _shadow_kv_to_cold(self, layer_idx: int, kv_layer: torch.Tensor, attn_metadata: Any,
                           store: ColdKVStore) -> None:
        new_tokens = (getattr(attn_metadata, "num_prefill_tokens", 0)
                      + getattr(attn_metadata, "num_decode_tokens", 0))
        if new_tokens == 0:
            return
        rows = _new_rows(kv_layer, new_tokens)
        if rows is None:
            logger.warning("unexpected kv_layer shape %s for layer %d; shadow copy skipped "
                           "(supported: [2, slots, H, D] and [2, blocks, block_size, H, D])",
                           tuple(kv_layer.shape), layer_idx)
            return
        store.evict_from_hot(*rows)

    def wait_for_save(self) -> None:
        """All layers of the step are saved: advance the decode step counter."""
        if self._prefill_complete:
            self._decode_step += 1

    def register_kv_caches(self, kv_caches: dict[str, torch.Tensor]) -> None:
        """vLLM's GPU cache buffers; the stores go on their device."""
        self._kv_caches = kv_caches
        if kv_caches:
            self._device = next(iter(kv_caches.values())).device

    def shutdown(self) -> None:
        self.cold_stores.clear()
        logger.info("KIVConnector shut down")

    # -- scheduler side -------------------------------------------------------------------------

    def get_num_new_matched_tokens(self, request: Any, num_computed_tokens: int) -> tuple[int | None, bool]:
        """KIV never supplies externally computed tokens."""
        return 0, False

    def update_state_after_alloc(self, request: Any, blocks: Any, num_external_tokens: int) -> None:
        """No per-request scheduler state."""

    def build_connector_meta(self, scheduler_output: Any) -> KIVConnectorMetadata:
        return KIVConnectorMetadata()

    @property
    def role(self) -> Any:
        return self._role

    @property
    def decode_step(self) -> int:
        """Decode steps completed since the first decode token."""
        return self._decode_step
