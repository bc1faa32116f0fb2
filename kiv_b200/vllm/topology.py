"""Model topology from a vLLM engine config (kiv/vllm/topology.py:17-193).

vLLM hands the connector its ``VllmConfig``; the HuggingFace config inside it
(``model_config.hf_config``, or its ``text_config`` for multimodal models)
carries everything the topology needs.  No model object is at hand, so the
rules read config fields only:

* global layers: the ``full_attention`` entries of ``layer_types`` (all layers
  when the list names none); otherwise every layer (a uniform
  ``sliding_window`` is managed as global too);
* KV sharing: with ``num_kv_shared_layers = s`` the global layers at or past
  ``num_hidden_layers - s`` reuse the KV of the last global layer before it;
* heads: ``num_global_key_value_heads`` / ``global_head_dim`` take priority
  over ``num_key_value_heads`` / ``head_dim``; MHA and
  ``hidden_size // heads`` are the fallbacks.
"""

from __future__ import annotations

import logging
from typing import Any

from ..model_topology import ModelTopology

logger = logging.getLogger(__name__)

_MODEL_TYPE_MAP = {
    "gemma4_text": "gemma4", "gemma4": "gemma4", "gemma3_text": "gemma3", "gemma3": "gemma3",
    "gemma3n_text": "gemma3n", "gemma3n": "gemma3n", "gemma2": "gemma2", "gemma": "gemma",
    "llama": "llama", "mistral": "mistral", "cohere2": "cohere2", "cohere": "cohere",
    "phi3": "phi3", "phi": "phi", "qwen2": "qwen2",
}


def _detect_global_layers(hf_config: Any) -> tuple[int, ...]:
    n = hf_config.num_hidden_layers
    layer_types = getattr(hf_config, "layer_types", None)
    if layer_types is not None:
        glob = tuple(i for i, t in enumerate(layer_types) if t == "full_attention")
        if glob:
            return glob
        logger.warning("layer_types names no full_attention layer; all %d layers treated as global", n)
        return tuple(range(n))
    if getattr(hf_config, "sliding_window", None) is not None:
        logger.info("uniform sliding_window: KIV manages all %d layers as global", n)
    return tuple(range(n))


def _detect_kv_sharing(hf_config: Any, global_indices: tuple[int, ...]) -> tuple[tuple[int, ...], dict[int, int]]:
    shared = getattr(hf_config, "num_kv_shared_layers", 0) or 0
    if shared <= 0:
        return tuple(global_indices), {}
    start = hf_config.num_hidden_layers - shared
    indep = tuple(i for i in global_indices if i < start)
    if not indep:
        return tuple(global_indices), {}
    return indep, {t: indep[-1] for t in global_indices if t >= start}


def _detect_head_geometry(hf_config: Any) -> tuple[int, int, int]:
    hq = hf_config.num_attention_heads
    hkv = getattr(hf_config, "num_global_key_value_heads", None)
    if hkv is None:
        hkv = getattr(hf_config, "num_key_value_heads", None)
    if hkv is None:
        hkv = hq
    d = getattr(hf_config, "global_head_dim", None)
    if d is None:
        d = getattr(hf_config, "head_dim", None)
    if d is None:
        d = hf_config.hidden_size // hq
    return hq, hkv, d


def detect_topology_from_vllm(vllm_config: Any) -> ModelTopology:
    """ModelTopology of the model a vLLM engine serves."""
    hf = vllm_config.model_config.hf_config
    if hasattr(hf, "text_config"):
        hf = hf.text_config
    model_type = getattr(hf, "model_type", "unknown")
    family = _MODEL_TYPE_MAP.get(model_type, model_type)
    if model_type not in _MODEL_TYPE_MAP:
        logger.warning("unknown model_type %r: all layers global, no KV sharing; pass a manual "
                       "topology for a better fit", model_type)
    glob = _detect_global_layers(hf)
    indep, sharing = _detect_kv_sharing(hf, glob)
    hq, hkv, d = _detect_head_geometry(hf)
    topo = ModelTopology(model_family=family, num_hidden_layers=hf.num_hidden_layers,
                         global_layer_indices=glob, independent_kv_layers=indep, kv_sharing_map=sharing,
                         num_query_heads=hq, num_kv_heads=hkv, head_dim=d)
    logger.info("KIV topology from vLLM config (%s): %d global layers (%d independent, %d shared), "
                "Hq %d, Hkv %d, D %d", family, len(glob), len(indep), len(sharing), hq, hkv, d)
    return topo
