"""Inference-side checkpoint loading (reference: tinytron/inference/checkpoint.py:25-92):
sharded training checkpoints are resharded into the inference layout (optionally
q/k/v-sharded by SEP rank) through the bridge; single-file state dicts go through
``state_dict_to_local_inference``."""
from __future__ import annotations

import os

import torch

from tinytron_b200.bridge import (BridgeContext, LayoutPlanner, ParallelSpec, RoutedMaterializer,
                                  StateDictShardFileStore, StateDictTensorStore, build_tinytron_canonical_layout,
                                  build_tinytron_inference_layout, build_tinytron_training_layout,
                                  current_tinytron_parallel_spec, current_tinytron_placement, localize_layout,
                                  state_dict_to_local_inference)


def checkpoint_prefix_from_model_path(model_path: str) -> str | None:
    if model_path.endswith("_model_canonical.pt"):
        return model_path[: -len("_model_canonical.pt")]
    if model_path.endswith("_model.pt"):
        return model_path[: -len("_model.pt")]
    if "_model_rank" in model_path and model_path.endswith(".pt"):
        return model_path.rsplit("_model_rank", 1)[0]
    return None


def checkpoint_meta_path(prefix: str) -> str:
    return f"{prefix}_meta.pt"


def checkpoint_model_shard_path(prefix: str, rank: int) -> str:
    return f"{prefix}_model_rank{rank:05d}.pt"


def load_model_state_dict_for_inference(checkpoint_path: str, model_config) -> dict[str, torch.Tensor]:
    prefix = checkpoint_prefix_from_model_path(checkpoint_path)
    if prefix is not None and os.path.exists(checkpoint_meta_path(prefix)):
        meta = torch.load(checkpoint_meta_path(prefix), map_location="cpu", weights_only=False)
        if bool(meta.get("model_sharded")) and os.path.exists(checkpoint_model_shard_path(prefix, 0)):
            return _reshard_from_files(prefix, model_config, meta)
    sd = torch.load(checkpoint_path, map_location="cpu", weights_only=True)
    return state_dict_to_local_inference(sd, model_config)


def _reshard_from_files(prefix: str, model_config, meta: dict):
    layout = meta.get("model_layout") or {}
    kind = layout.get("layout_kind", "canonical")
    if kind == "training":
        src = build_tinytron_training_layout(model_config, ParallelSpec(**layout.get("parallel", {})))
    elif kind == "canonical":
        src = build_tinytron_canonical_layout(model_config)
    else:
        raise ValueError(f"Unsupported checkpoint model layout kind: {kind}")
    dst = build_tinytron_inference_layout(model_config, current_tinytron_parallel_spec("inference"),
                                          shard_qkv=model_config.inference_shard_qkv)
    pl = current_tinytron_placement(dst)
    from tinytron_b200.training.checkpoint import verify_checksum

    class _Store(StateDictShardFileStore):
        def _sd(self, placement):
            verify_checksum(str(self.path_for_placement(placement)))
            return super()._sd(placement)

    store = _Store(lambda p: checkpoint_model_shard_path(prefix, int(p.rank or 0)))
    out = StateDictTensorStore()
    RoutedMaterializer().materialize(LayoutPlanner().plan(src, localize_layout(dst, pl)),
                                     BridgeContext(src_store=store, dst_store=out))
    return out.state_dict_for(pl)
