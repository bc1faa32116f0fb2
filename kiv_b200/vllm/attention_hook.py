"""Cold retrieval inside vLLM's attention layers (kiv/vllm/attention_hook.py:19-300).

``install_attention_hook(model, connector)`` wraps the inner ``Attention``
module's ``forward`` of every global layer: vLLM computes the hot output over
its own paged cache, then the wrapper runs the layer's cold retrieval and the
attention over the selected cold rows, and returns the equal-weight merge
``0.5 * hot + 0.5 * cold`` (the reference's merge; a log-sum-exp merge would
need the backend's softmax statistics).

Here the cold side is one fused path on the GPU: the store's coarse page
selection, fine token selection and the attention over the selected rows (the
store's own hot window is empty in connector mode, so ``ColdKVStore.attend``
attends over exactly the selected cold rows, as the reference's
``_cold_attention`` does over ``retrieve_top_kv``'s output).
"""

from __future__ import annotations

import logging
from typing import TYPE_CHECKING, Any

import torch

if TYPE_CHECKING:
    from .connector import KIVConnector

logger = logging.getLogger(__name__)


def _find_layers(model: Any) -> list[Any] | None:
    """The decoder layer list of a vLLM model."""
    for path in (lambda m: m.model.layers, lambda m: m.model.language_model.layers,
                 lambda m: m.model.text_model.layers, lambda m: m.layers):
        try:
            return list(path(model))
        except (AttributeError, TypeError):
            continue
    return None


def _find_self_attn(layer: Any) -> Any | None:
    for attr in ("self_attn", "attn", "attention"):
        mod = getattr(layer, attr, None)
        if mod is not None:
            return mod
    return None


def _find_inner_attn(self_attn: Any) -> Any | None:
    """vLLM's ``Attention`` object inside a model's attention module."""
    for attr in ("attn", "attention", "_attn"):
        obj = getattr(self_attn, attr, None)
        if obj is not None and hasattr(obj, "forward"):
            name = type(obj).__name__
            if "Attention" in name or "attn" in name.lower():
                return obj
    return None


def _query_bhqd(query: torch.Tensor, num_heads: int, head_dim: int) -> torch.Tensor | None:
    """vLLM query (``[T, H, D]``, ``[T, H*D]`` or ``[B, H, Q, D]``) as ``[B, H, Q, D]``."""
    if query.ndim == 3:
        return query.permute(1, 0, 2).unsqueeze(0)
    if query.ndim == 2:
        try:
            return query.view(query.shape[0], num_heads, head_dim).permute(1, 0, 2).unsqueeze(0)
        except RuntimeError:
            logger.debug("cannot view query %s as [T, %d, %d]", tuple(query.shape), num_heads, head_dim)
            return None
    if query.ndim == 4:
        return query
    logger.debug("unexpected query shape %s", tuple(query.shape))
    return None


def _as_hot_layout(cold_bqhd: torch.Tensor, target_shape: torch.Size) -> torch.Tensor | None:
    """Cold output ``[B, Q, H, D]`` (``attend``'s layout) in the hot output's layout
    (``[T, H*D]``, ``[T, H, D]`` or ``[B, H, Q, D]``), or None when it does not fit."""
    B, Q, H, D = cold_bqhd.shape
    target = tuple(target_shape)
    if len(target) == 4:
        out = cold_bqhd.transpose(1, 2)
    elif len(target) == 3:
        out = cold_bqhd.reshape(B * Q, H, D)
    elif len(target) == 2:
        out = cold_bqhd.reshape(B * Q, H * D)
    else:
        out = None
    if out is None or tuple(out.shape) != target:
        logger.debug("cannot lay cold output %s out as %s", tuple(cold_bqhd.shape), target)
        return None
    return out


def _make_kiv_inner_forward(original_forward: Any, layer_idx: int, connector: KIVConnector):
    """``Attention.forward`` wrapper: hot output from vLLM, cold output from the
    store's fused retrieval attention, equal-weight merge."""
    topo = connector.topology
    scaling = topo.head_dim ** -0.5

    def kiv_inner_forward(query, key, value, *args, **kwargs):
        hot = original_forward(query, key, value, *args, **kwargs)
        store = connector.get_cold_store(layer_idx)
        if store is None or store.cold_length == 0 or not connector._prefill_complete:
            return hot
        q = _query_bhqd(query, topo.num_query_heads, topo.head_dim)
        if q is None:
            return hot
        cold = store.attend(q, scaling, connector.kiv_config, step=connector._decode_step)
        cold = _as_hot_layout(cold, hot.shape)
        if cold is None:
            return hot
        if cold.dtype != hot.dtype:
            cold = cold.to(hot.dtype)
        return torch.lerp(hot, cold, 0.5)

    kiv_inner_forward.__wrapped__ = original_forward
    return kiv_inner_forward


def install_attention_hook(model: Any, connector: KIVConnector) -> dict[int, dict[str, Any]]:
    """Wrap the inner attention of every global layer of a vLLM model.

    Returns ``{layer_idx: {"inner_attn": module, "inner_forward": original}}``
    for ``uninstall_attention_hook``.  Layers without a separate inner
    ``Attention`` object are skipped (wrapping the outer module would recurse)."""
    originals: dict[int, dict[str, Any]] = {}
    layers = _find_layers(model)
    if layers is None:
        logger.warning("KIV attention hook: no layer list found on %s; cold retrieval is NOT active",
                       type(model).__name__)
        return originals
    for layer_idx in connector.topology.global_layer_indices:
        if layer_idx >= len(layers):
            continue
        self_attn = _find_self_attn(layers[layer_idx])
        if self_attn is None:
            continue
        inner = _find_inner_attn(self_attn)
        if inner is None or inner is self_attn:
            logger.debug("layer %d: no separate inner Attention object; skipped", layer_idx)
            continue
        original = inner.forward
        inner.forward = _make_kiv_inner_forward(original, layer_idx, connector)
        originals[layer_idx] = {"inner_attn": inner, "inner_forward": original}
    logger.info("KIV attention hooks installed on %d/%d global layers", len(originals),
                len(connector.topology.global_layer_indices))
    return originals


def uninstall_attention_hook(model: Any, originals: dict[int, dict[str, Any]]) -> None:
    """Put back the original inner ``forward`` methods."""
    for info in originals.values():
        info["inner_attn"].forward = info["inner_forward"]
    logger.info("KIV attention hooks removed from %d layers", len(originals))
