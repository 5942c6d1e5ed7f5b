"""Layout-aware checkpoint / weight-sync bridge (reference API: tinytron/bridge/__init__.py:18-49)."""
from __future__ import annotations

from .layout import LayoutIndex, Placement, RankCoord, ShardSpec, SliceSpec
from .planner import LayoutPlanner, TensorMove
from .rules import (ParallelSpec, build_tinytron_canonical_layout, build_tinytron_inference_layout,
                    build_tinytron_training_layout)

__all__ = [
    "BridgeContext", "DistributedCopyRoute", "DistributedStateDictStore", "LayoutIndex", "LayoutPlanner",
    "LocalCopyRoute", "P2PCopyRoute", "local_training_state_dict_to_local_inference", "localize_layout", "Placement",
    "RankCoord", "RoutedMaterializer", "ShardSpec", "SliceSpec", "FileTensorStore", "StateDictShardFileStore",
    "StateDictTensorStore", "state_dict_to_local_inference", "TensorMove", "TensorRoute", "TensorStore",
    "ParallelSpec", "build_tinytron_canonical_layout", "build_tinytron_inference_layout",
    "build_tinytron_training_layout", "bridge_metadata", "canonical_state_dict_to_local_inference",
    "canonical_state_dict_to_local_training", "current_tinytron_parallel_spec", "current_tinytron_placement",
    "distributed_training_state_dict_to_local_inference",
]

_LAZY = {
    "materializers": ("BridgeContext", "DistributedCopyRoute", "LocalCopyRoute", "P2PCopyRoute", "RoutedMaterializer",
                      "TensorRoute"),
    "stores": ("DistributedStateDictStore", "FileTensorStore", "StateDictShardFileStore", "StateDictTensorStore",
               "TensorStore"),
    "model": ("bridge_metadata", "canonical_state_dict_to_local_inference", "canonical_state_dict_to_local_training",
              "current_tinytron_parallel_spec", "current_tinytron_placement",
              "distributed_training_state_dict_to_local_inference", "local_training_state_dict_to_local_inference",
              "localize_layout", "state_dict_to_local_inference"),
}


def __getattr__(name: str):
    import importlib

    for mod, names in _LAZY.items():
        if name in names:
            return getattr(importlib.import_module(f"{__name__}.{mod}"), name)
    raise AttributeError(f"module {__name__!r} has no attribute {name!r}")
