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
    # Pinned host overflow tier: cold tokens per layer kept in host memory once
    # the HBM cold tier (cold_capacity tokens, then a ring of the newest pages)
    # is full.  0: no host tier (the cold tier grows in HBM).  Needs cold_capacity.
    host_tokens: int = 0
    # HBM staging pages for the host-resident pages of one retrieval's union.
    stage_pages: int = 1024

    def __post_init__(self) -> None:
        if self.host_tokens < 0 or self.stage_pages < 1:
            raise ValueError("host_tokens must be >= 0 and stage_pages >= 1")
        if self.host_tokens > 0 and not self.cold_capacity:
            raise ValueError("a host tier (host_tokens > 0) needs cold_capacity (the HBM ring size)")
