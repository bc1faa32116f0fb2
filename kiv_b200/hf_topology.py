"""Detect a ``ModelTopology`` from a loaded HuggingFace model.

Behaviour follows the reference's ``kiv/hf_topology.py:13-225``: global layers
from ``layer_types`` (else every layer), KV sharing from
``num_kv_shared_layers`` or per-module ``is_kv_shared_layer`` flags, head
geometry preferring the global-layer fields (Gemma-4 style).
"""

from __future__ import annotations

import logging
from typing import Any

from .model_topology import ModelTopology

logger = logging.getLogger(__name__)

_FAMILIES = {
    "gemma4_text": "gemma4", "gemma4": "gemma4",
    "gemma3_text": "gemma3", "gemma3": "gemma3",
    "gemma3n_text": "gemma3n", "gemma3n": "gemma3n",
    "gemma2": "gemma2", "gemma": "gemma",
    "llama": "llama", "mistral": "mistral",
    "cohere2": "cohere2", "cohere": "cohere",
    "phi3": "phi3", "phi": "phi",
    "qwen2": "qwen2",
}


def _resolve_text_config(model: Any) -> Any:
    cfg = model.config
    return cfg.text_config if hasattr(cfg, "text_config") else cfg


def _find_text_model(model: Any) -> Any:
    """The module that holds ``.layers`` (multimodal wrappers unwrapped)."""
    inner = getattr(model, "model", None)
    if inner is not None:
        for name in ("language_model", "text_model"):
            sub = getattr(inner, name, None)
            if sub is not None and hasattr(sub, "layers"):
                return sub
        if hasattr(inner, "layers"):
            return inner
    raise AttributeError("Cannot find text model layers. Supported: model.model.language_model, "
                         "model.model.text_model, model.model")


def _detect_global_layers(config: Any) -> tuple[int, ...]:
    n = config.num_hidden_layers
    layer_types = getattr(config, "layer_types", None)
    if layer_types is not None:
        full = tuple(i for i, t in enumerate(layer_types) if t == "full_attention")
        if full:
            return full
        logger.warning("layer_types has no 'full_attention' entry; treating all %d layers as global", n)
        return tuple(range(n))
    if getattr(config, "sliding_window", None) is not None:
        logger.info("uniform sliding_window: KIV manages all %d layers as global", n)
    return tuple(range(n))


def _detect_kv_sharing(config: Any, model: Any, global_indices: tuple[int, ...]):
    n = config.num_hidden_layers
    shared = getattr(config, "num_kv_shared_layers", 0) or 0
    if shared > 0:
        first_shared = n - shared
        indep = tuple(i for i in global_indices if i < first_shared)
        targets = tuple(i for i in global_indices if i >= first_shared)
        if not indep:
            return global_indices, {}
        return indep, {t: indep[-1] for t in targets}
    try:
        layers = _find_text_model(model).layers
        indep, sharing = [], {}
        for i in global_indices:
            attn = layers[i].self_attn
            src = getattr(attn, "kv_shared_layer_index", None)
            if getattr(attn, "is_kv_shared_layer", False) and src is not None:
                sharing[i] = src
            else:
                indep.append(i)
        if sharing:
            return tuple(indep), sharing
    except (AttributeError, IndexError):
        pass
    return global_indices, {}


def _detect_head_geometry(config: Any) -> tuple[int, int, int]:
    hq = config.num_attention_heads
    hkv = getattr(config, "num_global_key_value_heads", None)
    if hkv is None:
        hkv = getattr(config, "num_key_value_heads", None)
    if hkv is None:
        hkv = hq
    d = getattr(config, "global_head_dim", None)
    if d is None:
        d = getattr(config, "head_dim", None)
    if d is None:
        d = config.hidden_size // hq
    return hq, hkv, d


def detect_topology(model: Any) -> ModelTopology:
    """Build the topology of a HuggingFace model (unknown families: all layers global, no sharing)."""
    config = _resolve_text_config(model)
    model_type = getattr(config, "model_type", "unknown")
    family = _FAMILIES.get(model_type)
    if family is None:
        logger.warning("Unknown model_type '%s'. Treating all layers as global with no KV sharing. "
                       "Pass a manual ModelTopology for better efficiency.", model_type)
        family = model_type
    glob = _detect_global_layers(config)
    indep, sharing = _detect_kv_sharing(config, model, glob)
    hq, hkv, d = _detect_head_geometry(config)
    topo = ModelTopology(model_family=family, num_hidden_layers=config.num_hidden_layers,
                         global_layer_indices=glob, independent_kv_layers=indep,
                         kv_sharing_map=sharing, num_query_heads=hq, num_kv_heads=hkv, head_dim=d)
    logger.info("KIV topology for %s: %d global layers (%d independent, %d shared), "
                "%d query heads, %d KV heads, head_dim=%d", family, len(glob), len(indep),
                len(sharing), hq, hkv, d)
    return topo
