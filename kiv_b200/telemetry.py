"""Retrieval telemetry without host syncs on the decode path.

Same record kinds, keys and aggregates as the reference's ``_RetrievalTelemetry``
(kiv/cold_store.py:417-580).  The reference calls ``.cpu()`` five times per
retrieval; here each call only launches small device-to-device copies of the
kernel-computed values (union pages, selected token ids, max / sum of the
coarse and fine scores); everything is materialized on ``snapshot()``.
"""

from __future__ import annotations

import struct
from dataclasses import dataclass

import torch

from . import _native as nat

MAX_RECORDS = 256


def _key_to_float(key: int) -> float:
    """Invert the kernels' order-preserving float -> uint32 key."""
    k = key & 0xFFFFFFFF
    u = (k & 0x7FFFFFFF) if (k & 0x80000000) else (~k & 0xFFFFFFFF)
    return struct.unpack("<f", struct.pack("<I", u))[0]


def _bits_to_double(word: int) -> float:
    return struct.unpack("<d", struct.pack("<q", word))[0]


@dataclass
class _Pending:
    kind: str
    cold_length: int
    num_pages: int = 0
    skipped: bool = False
    pages: torch.Tensor | None = None       # device int32, first `count` valid
    tokens: torch.Tensor | None = None      # device int32 [B, P]
    stats: torch.Tensor | None = None       # device int64 copy of state words
    n_scores: int = 0
    actual_P: int = 0
    requested_P: int = 0


class RetrievalTelemetry:
    """Ring of the last ``MAX_RECORDS`` coarse / fine records plus running aggregates."""

    _MAX_BUFFER = MAX_RECORDS

    def __init__(self, enabled: bool = True) -> None:
        self.enabled = enabled
        self._pending: list[_Pending] = []
        self._ring: list[dict] = []
        self.total_calls = 0
        self.coarse_calls = 0
        self.coarse_real_calls = 0
        self.coarse_top_score_sum = 0.0
        self.coarse_mean_score_sum = 0.0
        self.coarse_cold_length_sum = 0
        self.fine_calls = 0
        self.fine_top_score_sum = 0.0
        self.fine_mean_score_sum = 0.0
        self.selected_count_sum = 0

    # -- recording (no host sync) --
    def record_coarse(self, *, state: torch.Tensor, union: torch.Tensor, num_pages: int,
                      cold_length: int, n_scores: int) -> None:
        if not self.enabled:
            return
        self._pending.append(_Pending("coarse", cold_length, num_pages, False, union.clone(), None,
                                      state[nat.ST_UNION:nat.ST_FINE_MAX].clone(), n_scores))
        self._trim()

    def record_coarse_skipped(self, *, cold_length: int) -> None:
        if not self.enabled:
            return
        self._pending.append(_Pending("coarse", cold_length, 0, True))
        self._trim()

    def record_fine(self, *, state: torch.Tensor, selected: torch.Tensor, actual_P: int,
                    requested_P: int, cold_length: int, n_scores: int) -> None:
        if not self.enabled:
            return
        self._pending.append(_Pending("fine", cold_length, 0, False, None, selected.clone(),
                                      state[nat.ST_CAND:nat.ST_FINE_SUM + 1].clone(), n_scores,
                                      actual_P, requested_P))
        self._trim()

    def _trim(self) -> None:
        if len(self._pending) > 4 * MAX_RECORDS:
            self._flush()

    # -- materialization --
    def _flush(self) -> None:
        for p in self._pending:
            if p.kind == "coarse" and p.skipped:
                self.coarse_calls += 1
                self.coarse_cold_length_sum += p.cold_length
                self._push({"kind": "coarse", "cold_length": p.cold_length, "num_pages": 0,
                            "num_pages_selected": 0, "top_score": 0.0, "mean_score": 0.0,
                            "score_ratio": 0.0, "pages_selected": [], "skipped": True})
            elif p.kind == "coarse":
                st = p.stats.cpu().tolist()           # words UNION .. COARSE_SUM
                u = int(st[0])
                top = _key_to_float(int(st[nat.ST_COARSE_MAX - nat.ST_UNION]))
                total = _bits_to_double(int(st[nat.ST_COARSE_SUM - nat.ST_UNION]))
                mean = total / max(p.n_scores, 1)
                pages = p.pages[:u].cpu().tolist()
                self.coarse_calls += 1
                self.coarse_real_calls += 1
                self.coarse_top_score_sum += top
                self.coarse_mean_score_sum += mean
                self.coarse_cold_length_sum += p.cold_length
                self._push({"kind": "coarse", "cold_length": p.cold_length,
                            "num_pages": p.num_pages, "num_pages_selected": len(pages),
                            "top_score": top, "mean_score": mean,
                            "score_ratio": (top / abs(mean)) if mean else float("inf"),
                            "pages_selected": pages, "skipped": False})
            else:
                st = p.stats.cpu().tolist()           # words CAND .. FINE_SUM
                cand = int(st[0])
                top = _key_to_float(int(st[nat.ST_FINE_MAX - nat.ST_CAND]))
                total = _bits_to_double(int(st[nat.ST_FINE_SUM - nat.ST_CAND]))
                mean = total / max(p.tokens.shape[0] * cand, 1)
                sel = p.tokens[:, :p.actual_P].reshape(-1).cpu().tolist()
                self.fine_calls += 1
                self.total_calls += 1
                self.fine_top_score_sum += top
                self.fine_mean_score_sum += mean
                self.selected_count_sum += p.actual_P
                self._push({"kind": "fine", "cold_length": p.cold_length, "actual_P": p.actual_P,
                            "requested_P": p.requested_P, "top_score": top, "mean_score": mean,
                            "score_ratio": (top / abs(mean)) if mean else float("inf"),
                            "selected_token_indices": sel})
        self._pending.clear()

    def _push(self, rec: dict) -> None:
        self._ring.append(rec)
        if len(self._ring) > self._MAX_BUFFER:
            self._ring = self._ring[-self._MAX_BUFFER:]

    def snapshot(self) -> dict:
        """Aggregates and recent records, in the reference's format (syncs the device)."""
        self._flush()
        agg = {"total_calls": self.total_calls, "coarse_calls": self.coarse_calls,
               "coarse_real_calls": self.coarse_real_calls,
               "coarse_skipped_calls": self.coarse_calls - self.coarse_real_calls,
               "fine_calls": self.fine_calls}
        if self.coarse_real_calls:
            agg["avg_coarse_top_score"] = self.coarse_top_score_sum / self.coarse_real_calls
            agg["avg_coarse_mean_score"] = self.coarse_mean_score_sum / self.coarse_real_calls
        if self.coarse_calls:
            agg["avg_cold_length"] = self.coarse_cold_length_sum / self.coarse_calls
        if self.fine_calls:
            agg["avg_fine_top_score"] = self.fine_top_score_sum / self.fine_calls
            agg["avg_fine_mean_score"] = self.fine_mean_score_sum / self.fine_calls
            agg["avg_selected_P"] = self.selected_count_sum / self.fine_calls
        return {"aggregates": agg, "recent": list(self._ring)}
