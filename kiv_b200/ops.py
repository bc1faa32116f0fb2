"""``torch.ops.kiv.*``: the C ABI of ``libkiv_b200.so`` registered with PyTorch.

``_kiv_ops.so`` (built from ``csrc/torch_ops.cpp`` next to the CUDA library)
registers one operator per compute entry point of ``include/kiv_b200.h``
under the ``kiv`` namespace, with a CUDA kernel that calls the entry point on
the current stream and a Meta kernel for tracing with fake tensors.  The
cold store calls the kernels through these operators; ``_native`` (ctypes)
remains for the host-only calls (peer and pinned-host allocation, exchange
sizing) and for tests of the raw ABI.

A store crosses as ``(store, geom)``: nine tensors ``[cold_k, cold_v,
summaries, hot_k, hot_v, state, host_k, host_v, page_sums]`` (empty tensors
for a missing hot ring, host tier or running page sums) and six ints
``[page_size, shard_rank, shard_count, hot_hint, stage_pages, flags]``.
There is no fallback: a missing operator library raises.
"""

from __future__ import annotations

import os
import threading

import torch

from . import _native as nat

HERE = os.path.dirname(os.path.abspath(__file__))
OPS_PATH = os.path.join(HERE, "_kiv_ops.so")

_loaded = False
_lock = threading.Lock()


def load() -> None:
    """Load the CUDA library and register ``torch.ops.kiv`` (once)."""
    global _loaded
    with _lock:
        if _loaded:
            return
        nat.load_library()
        if not os.path.exists(OPS_PATH):
            raise nat.KIVNativeError(
                f"{OPS_PATH} not found; build it with `python -c 'import __graft_entry__ as g; g.build()'` "
                "(make -C kiv_b200/csrc)")
        try:
            torch.ops.load_library(OPS_PATH)
        except OSError as e:  # pragma: no cover - depends on the machine
            raise nat.KIVNativeError(f"cannot load {OPS_PATH}: {e}") from e
        _loaded = True


def kiv():
    """The ``torch.ops.kiv`` namespace (loads it on first use)."""
    if not _loaded:
        load()
    return torch.ops.kiv


def call(op, *args):
    """Run an operator; library failures surface as KIVNativeError."""
    try:
        return op(*args)
    except RuntimeError as e:
        if "kiv." in str(e) or "kiv:" in str(e):
            raise nat.KIVNativeError(str(e)) from e
        raise


OP_NAMES = ("state_reset", "append_evict", "workspace_layout", "coarse_select", "coarse_merge", "fine_score",
            "fine_topk", "fine_select", "fine_merge", "gather_rows", "attend", "attend_merge", "retrieve_attend",
            "coarse_exchange_merge", "fine_exchange_merge", "attend_exchange_merge", "fine_exchange_select",
            "attend_peers")
