"""vLLM integration (kiv/vllm/__init__.py): a V1 KV connector that shadows each
global layer's new K/V rows into GPU cold stores, and an attention hook that
adds cold retrieval to vLLM's attention layers.  Importing this package does
not import vLLM; the connector subclasses ``KVConnectorBase_V1`` when vLLM is
importable."""

from .attention_hook import install_attention_hook, uninstall_attention_hook
from .connector import KIVConnector, KIVConnectorMetadata
from .topology import detect_topology_from_vllm

__all__ = ["KIVConnector", "KIVConnectorMetadata", "install_attention_hook", "uninstall_attention_hook",
           "detect_topology_from_vllm"]
