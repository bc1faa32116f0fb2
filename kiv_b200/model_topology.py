"""Model geometry that KIV needs: which layers are global, which share KV, head shapes.

Same fields, invariants and ``manual`` constructor as the reference's
``kiv/model_topology.py:9-85``.
"""

from __future__ import annotations

from dataclasses import dataclass, field


@dataclass(frozen=True)
class ModelTopology:
    """Frozen descriptor of the attention layers KIV manages.

    Invariants checked at construction:
    * every independent KV layer is a global layer;
    * every KV-sharing layer (a key of ``kv_sharing_map``) is a global layer;
    * every sharing source (a value of ``kv_sharing_map``) owns a cold store,
      i.e. is an independent KV layer.
    """

    model_family: str
    num_hidden_layers: int
    global_layer_indices: tuple[int, ...]
    independent_kv_layers: tuple[int, ...]
    kv_sharing_map: dict[int, int] = field(default_factory=dict)
    num_query_heads: int = 0
    num_kv_heads: int = 0
    head_dim: int = 0

    def __post_init__(self) -> None:
        glob = set(self.global_layer_indices)
        indep = set(self.independent_kv_layers)
        extra = indep - glob
        if extra:
            raise ValueError("independent_kv_layers must be a subset of global_layer_indices; "
                             f"extras: {sorted(extra)}")
        extra = set(self.kv_sharing_map) - glob
        if extra:
            raise ValueError("kv_sharing_map keys must all appear in global_layer_indices; "
                             f"extras: {sorted(extra)}")
        extra = set(self.kv_sharing_map.values()) - indep
        if extra:
            raise ValueError("kv_sharing_map values must all appear in independent_kv_layers; "
                             f"extras: {sorted(extra)}")

    @staticmethod
    def manual(*, global_layer_indices: tuple[int, ...], num_query_heads: int, num_kv_heads: int,
               head_dim: int, num_hidden_layers: int,
               independent_kv_layers: tuple[int, ...] | None = None,
               kv_sharing_map: dict[int, int] | None = None,
               model_family: str = "unknown") -> "ModelTopology":
        """Build a topology by hand (independent layers default to all global layers)."""
        return ModelTopology(
            model_family=model_family,
            num_hidden_layers=num_hidden_layers,
            global_layer_indices=tuple(global_layer_indices),
            independent_kv_layers=tuple(global_layer_indices if independent_kv_layers is None
                                        else independent_kv_layers),
            kv_sharing_map=dict(kv_sharing_map or {}),
            num_query_heads=num_query_heads,
            num_kv_heads=num_kv_heads,
            head_dim=head_dim,
        )
