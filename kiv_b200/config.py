"""KIV algorithm and budget knobs (same fields and defaults as the reference's
``kiv/config.py:7-26``), plus optional capacity knobs of the HBM-resident tiers."""

from dataclasses import dataclass


@dataclass
class KIVConfig:
    """Tunable parameters of K-Indexed V materialization.

    The first five fields are the reference's and keep its defaults, so every
    existing constructor call keeps working.  The rest are optional and only
    concern where the tiers live on a B200.
    """

    # exact K/V kept for the most recent tokens
    hot_budget: int = 2048
    # cold tokens retrieved per step
    top_p: int = 256
    # coarse-to-fine retrieval geometry
    page_size: int = 128
    top_pages: int = 32
    # Accepted for compatibility.  The cold tier is HBM-resident here, so there
    # is no host fetch to overlap; the flag is kept but has no effect.
    prefetch_stream: bool = True

    # Cold-tier token slots to preallocate per layer (None: grow on demand by
    # doubling).  Preallocating keeps device pointers fixed, which a captured
    # CUDA graph of the decode step needs.
    cold_capacity: int | None = None
    # Extra hot-window rows beyond hot_budget before the window is compacted.
    hot_slack: int = 2048
    # Record per-call retrieval telemetry (copied asynchronously, no host sync).
    telemetry: bool = True
