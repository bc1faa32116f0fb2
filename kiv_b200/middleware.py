"""KIV middleware for HuggingFace transformers.

Drop-in for the reference's ``KIVMiddleware`` (kiv/middleware.py:43-356):
``install()`` registers ``kiv_<impl>`` in ``ALL_ATTENTION_FUNCTIONS`` (and
mirrors the mask function), ``create_cache()`` / ``activate_cache()`` bind a
``TieredKVCache``, ``chunked_prefill()`` runs chunks with the native attention.

The attention wrapper differs in what it calls: where the reference retrieves
cold K/V, concatenates ``[cold ; hot]``, extends the mask and calls the
original attention, this wrapper calls the fused retrieval-attention kernels
(``ColdKVStore.attend``), which read the selected cold rows in place and the
hot window from the cache.  With no cold tokens (or cold suppressed) it calls
the original attention function, exactly as the reference does.
"""

from __future__ import annotations

import importlib
import inspect
import logging
from typing import Any

import torch
from transformers.masking_utils import ALL_MASK_ATTENTION_FUNCTIONS
from transformers.modeling_utils import ALL_ATTENTION_FUNCTIONS

from .config import KIVConfig
from .hf_topology import _find_text_model, detect_topology
from .mask_utils import extend_mask_for_cold
from .model_topology import ModelTopology
from .tiered_cache import TieredKVCache

logger = logging.getLogger(__name__)

_extend_mask_for_cold = extend_mask_for_cold


def invalidate_cold_candidate_caches(cache: Any) -> None:
    """Drop every cold store's per-step candidate reuse (kiv/server/generation.py:183-197)."""
    for store in (getattr(cache, "cold_stores", None) or {}).values():
        store._cached_candidate_k = None
        store._cached_candidate_v = None
        store._cached_candidate_idx = None
        store._cached_step = -1


def chunked_reuse_prefill(model: Any, input_ids: torch.Tensor, cache: Any, *, chunk_size: int = 4096) -> torch.Tensor:
    """Prefill a prompt tail chunk by chunk WITH cold retrieval on every chunk
    (the reference server's reuse prefill, kiv/server/generation.py:123-180):
    inside a chunk nothing is evicted (the chunk's later positions still attend
    to its earlier ones in the hot window) and the per-step candidate caches
    are dropped first (no decode step advances inside a chunk); between chunks
    the hot overflow moves to the cold tier.  The attention of every chunk goes
    through the KIV wrapper, i.e. the prefill-shaped retrieval kernels.
    Returns the last position's logits ``[B, vocab]``."""
    total = input_ids.shape[1]
    last = None
    prior = getattr(cache, "_prefill_complete", True)
    try:
        with torch.no_grad():
            for a in range(0, total, chunk_size):
                b = min(a + chunk_size, total)
                invalidate_cold_candidate_caches(cache)
                cache._prefill_complete = False
                out = model(input_ids=input_ids[:, a:b], past_key_values=cache, use_cache=True)
                if b == total:
                    last = out.logits[:, -1, :].clone()
                del out
                cache._prefill_complete = True
                if hasattr(cache, "_evict_excess_all_layers"):
                    cache._evict_excess_all_layers()
    finally:
        cache._prefill_complete = prior
    if last is None:
        raise RuntimeError("prefill produced no logits")
    return last


def _prefill_logits_kwargs(model: Any, logits_to_keep: int = 1) -> dict[str, int]:
    """``{"logits_to_keep": n}`` when the model's forward accepts it (feature-detected)."""
    try:
        params = inspect.signature(model.forward).parameters
    except (TypeError, ValueError, AttributeError):
        return {}
    return {"logits_to_keep": logits_to_keep} if "logits_to_keep" in params else {}


def hot_mask_for_kernel(attention_mask: torch.Tensor | None, hot_len: int, q_len: int):
    """Translate an HF attention mask into the kernel's hot-window mask.

    Returns ``(additive float32 mask [B, 1|H, Q, hot_len] or None, causal)``.
    The mask is cropped to its last ``hot_len`` columns (it was built before
    this step's eviction, kiv/middleware.py:333-340); the cold columns need no
    mask (all attendable, kiv/mask_utils.py:8-38).  No mask with Q > 1 means
    causal, the convention of HF's sdpa / flash paths.
    """
    if attention_mask is None:
        return None, q_len > 1
    m = attention_mask
    if m.shape[-1] > hot_len:
        m = m[..., -hot_len:]
    causal = False
    if m.dim() == 2:  # padding mask [B, KV] (1 / True = attend)
        m = m[:, None, None, :]
        causal = q_len > 1
    if m.dtype == torch.bool or not m.dtype.is_floating_point:
        m = torch.where(m.bool(), 0.0, float("-inf")).to(torch.float32)
    elif m.dtype != torch.float32:
        m = m.float()
    if m.shape[-2] != q_len:
        m = m.expand(m.shape[0], m.shape[1], q_len, m.shape[-1])
    if m.stride(-1) != 1:
        m = m.contiguous()
    return m, causal


class KIVMiddleware:
    """Installs KIV's retrieval attention into a HuggingFace model."""

    def __init__(self, model: Any, config: KIVConfig | None = None,
                 topology: ModelTopology | None = None) -> None:
        self.model = model
        self.config = config or KIVConfig()
        self._topology_override = topology
        self.topology: ModelTopology | None = None
        self._text_model: Any = None
        self._installed = False
        self._original_impl: str | None = None
        self._kiv_key: str | None = None

    def install(self) -> None:
        if self._installed:
            logger.warning("KIV middleware already installed.")
            return
        if self._topology_override is not None:
            self.topology = self._topology_override
            logger.info("Using manually provided ModelTopology.")
        else:
            self.topology = detect_topology(self.model)
        self._text_model = _find_text_model(self.model)
        for li in self.topology.global_layer_indices:
            self._text_model.layers[li].self_attn._kiv_layer_idx = li
        self._original_impl = self._resolve_attn_impl()
        original_fn = self._get_attn_fn(self._original_impl)
        self._kiv_key = f"kiv_{self._original_impl}"
        ALL_ATTENTION_FUNCTIONS[self._kiv_key] = self._make_kiv_attention(original_fn)
        # _preprocess_mask_arguments reads _global_mapping directly
        if self._original_impl in ALL_MASK_ATTENTION_FUNCTIONS:
            ALL_MASK_ATTENTION_FUNCTIONS._global_mapping[self._kiv_key] = (
                ALL_MASK_ATTENTION_FUNCTIONS[self._original_impl])
        self._set_attn_impl(self._kiv_key)
        self._installed = True
        logger.info("KIV middleware installed: %d global layers (%d independent, %d shared), "
                    "attn=%s, hot=%d, top_p=%d", len(self.topology.global_layer_indices),
                    len(self.topology.independent_kv_layers), len(self.topology.kv_sharing_map),
                    self._original_impl, self.config.hot_budget, self.config.top_p)

    def uninstall(self) -> None:
        if not self._installed:
            return
        if self._original_impl is not None:
            self._set_attn_impl(self._original_impl)
        if self._kiv_key is not None:
            if self._kiv_key in ALL_ATTENTION_FUNCTIONS:
                del ALL_ATTENTION_FUNCTIONS[self._kiv_key]
            ALL_MASK_ATTENTION_FUNCTIONS._global_mapping.pop(self._kiv_key, None)
        if self._text_model is not None and self.topology is not None:
            for li in self.topology.global_layer_indices:
                attn = self._text_model.layers[li].self_attn
                for attr in ("_kiv_layer_idx", "_kiv_cache"):
                    if hasattr(attn, attr):
                        delattr(attn, attr)
        self._installed = False
        self._original_impl = None
        self._kiv_key = None
        logger.info("KIV middleware uninstalled.")

    def create_cache(self, device: torch.device | None = None, *, shard_group=None,
                     batch_group=None) -> TieredKVCache:
        """``shard_group``: split every layer's cold pages over the group's ranks
        (one sequence, strong scaling); ``batch_group``: this rank holds its own
        sequences of the batch and the page union is taken over the group."""
        if self.topology is None:
            raise RuntimeError("Call install() before create_cache().")
        if device is None:
            device = next(self.model.parameters()).device
        cache = TieredKVCache(config=self.model.config, kiv_config=self.config,
                              topology=self.topology, device=device, shard_group=shard_group,
                              batch_group=batch_group)
        self.activate_cache(cache)
        return cache

    def activate_cache(self, cache: TieredKVCache | None) -> None:
        """Point the attention wrapper of every global layer at ``cache``."""
        if self.topology is None or self._text_model is None:
            return
        for li in self.topology.global_layer_indices:
            attn = self._text_model.layers[li].self_attn
            if cache is None:
                if hasattr(attn, "_kiv_cache"):
                    delattr(attn, "_kiv_cache")
            else:
                attn._kiv_cache = cache

    def chunked_prefill(self, input_ids: torch.Tensor, cache: TieredKVCache, chunk_size: int = 4096,
                        prefill_hot_cap: int | None = None,
                        empty_cache_interval: int | None = None) -> torch.Tensor:
        """Prefill a long prompt chunk by chunk with the native attention (no
        retrieval), optionally capping the hot window between chunks; returns the
        last position's logits ``[B, vocab]`` (kiv/middleware.py:174-260)."""
        if not self._installed:
            raise RuntimeError("Call install() before chunked_prefill().")
        _, T = input_ids.shape
        n_chunks = (T + chunk_size - 1) // chunk_size
        logits = None
        extra = _prefill_logits_kwargs(self.model, logits_to_keep=1)
        if prefill_hot_cap is not None:
            cache._suppress_cold = True
        self._set_attn_impl(self._original_impl)
        try:
            for i in range(n_chunks):
                a, b = i * chunk_size, min((i + 1) * chunk_size, T)
                with torch.no_grad():
                    out = self.model(input_ids=input_ids[:, a:b], past_key_values=cache,
                                     use_cache=True, **extra)
                if b == T:
                    logits = out.logits[:, -1, :]
                del out
                if prefill_hot_cap is not None:
                    cache._evict_to_cap(prefill_hot_cap)
                if empty_cache_interval and empty_cache_interval > 0 and (i + 1) % empty_cache_interval == 0:
                    torch.cuda.empty_cache()
        finally:
            cache._suppress_cold = False
            self._set_attn_impl(self._kiv_key)
        if prefill_hot_cap is None:
            cache.mark_prefill_complete()
        else:
            cache._prefill_complete = True
            cache._evict_excess_all_layers()
        return logits

    def chunked_retrieval_prefill(self, input_ids: torch.Tensor, cache: TieredKVCache,
                                  chunk_size: int = 4096) -> torch.Tensor:
        """Prefill with cold retrieval on every chunk (see ``chunked_reuse_prefill``);
        the KIV attention stays installed, so each chunk retrieves from the cold tier."""
        if not self._installed:
            raise RuntimeError("Call install() before chunked_retrieval_prefill().")
        return chunked_reuse_prefill(self.model, input_ids, cache, chunk_size=chunk_size)

    def _resolve_attn_impl(self) -> str:
        cfg = self.model.config
        if hasattr(cfg, "text_config"):
            cfg = cfg.text_config
        return getattr(cfg, "_attn_implementation", "eager")

    def _get_attn_fn(self, impl: str) -> Any:
        if impl in ALL_ATTENTION_FUNCTIONS:
            return ALL_ATTENTION_FUNCTIONS[impl]
        attn = self._text_model.layers[self.topology.global_layer_indices[0]].self_attn
        fn = getattr(importlib.import_module(type(attn).__module__), "eager_attention_forward", None)
        if fn is not None:
            return fn
        raise ValueError(f"Cannot find attention function for implementation '{impl}'")

    def _set_attn_impl(self, impl: str) -> None:
        cfg = self.model.config
        if hasattr(cfg, "text_config"):
            cfg.text_config._attn_implementation = impl
        cfg._attn_implementation = impl

    def _make_kiv_attention(self, original_fn: Any) -> Any:
        kiv_config = self.config
        sample = self._text_model.layers[self.topology.global_layer_indices[0]].self_attn
        fallback_scaling = (sample.scaling if getattr(sample, "scaling", None) is not None
                            else self.topology.head_dim ** -0.5)

        def kiv_attention(module, query, key, value, attention_mask, **kwargs):
            cache = getattr(module, "_kiv_cache", None)
            layer_idx = getattr(module, "_kiv_layer_idx", None)
            if cache is not None and layer_idx is not None:
                store = cache.get_cold_store(layer_idx)
                if (store is not None and store.cold_length > 0
                        and not getattr(cache, "_suppress_cold", False)
                        and key.shape[2] == store.hot_length):
                    scaling = kwargs.get("scaling")
                    if scaling is None:
                        scaling = fallback_scaling
                    mask_add, causal = hot_mask_for_kernel(attention_mask, store.hot_length,
                                                           query.shape[2])
                    out = store.attend(query, scaling, kiv_config,
                                       step=getattr(cache, "_decode_step", -1), mask_add=mask_add,
                                       causal=causal, softcap=kwargs.get("softcap"))
                    return out.to(query.dtype), None
            return original_fn(module, query, key, value, attention_mask, **kwargs)

        return kiv_attention
