"""Attention-mask helper (same contract as the reference's ``kiv/mask_utils.py:8-38``).

The fused attention kernel never needs this -- cold columns are always
attendable, so it reads only the hot part of the mask -- but callers that
concatenate cold K/V themselves (the ``retrieve_top_kv`` API) still do.
"""

from __future__ import annotations

import torch


def extend_mask_for_cold(mask: torch.Tensor, num_cold: int) -> torch.Tensor:
    """Prepend ``num_cold`` all-attendable columns on the last dim.

    Boolean masks get ``True`` (attend), additive float masks get ``0.0``; the
    leading dims of the mask are kept (``[B, KV]``, ``[B, H, Q, KV]`` or any).
    """
    fill = True if mask.dtype == torch.bool else 0.0
    cols = mask.new_full(tuple(mask.shape[:-1]) + (num_cold,), fill)
    return torch.cat([cols, mask], dim=-1)
