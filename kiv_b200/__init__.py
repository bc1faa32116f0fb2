"""kiv_b200: B200-native (sm_100a) KIV tiered-cache retrieval attention.

Same public surface as the reference package ``kiv``: ``KIVConfig``,
``ColdKVStore``, ``ModelTopology``, ``detect_topology``, ``TieredKVCache``,
``KIVMiddleware``.  The heavy imports (transformers) are lazy, like the reference.
"""

__version__ = "0.1.0"

from .config import KIVConfig
from .model_topology import ModelTopology

__all__ = ["KIVConfig", "ColdKVStore", "ModelTopology", "detect_topology", "TieredKVCache",
           "KIVMiddleware"]


def __getattr__(name: str):
    if name == "ColdKVStore":
        from .cold_store import ColdKVStore
        return ColdKVStore
    if name == "detect_topology":
        from .hf_topology import detect_topology
        return detect_topology
    if name == "TieredKVCache":
        from .tiered_cache import TieredKVCache
        return TieredKVCache
    if name == "KIVMiddleware":
        from .middleware import KIVMiddleware
        return KIVMiddleware
    raise AttributeError(f"module 'kiv_b200' has no attribute {name!r}")
