"""Model-level bridge helpers (reference: tinytron/bridge/model.py:24-257): the live
parallel spec / placement, metadata for checkpoints, and state-dict conversions
canonical <-> training <-> inference."""
from __future__ import annotations

from dataclasses import asdict

import torch
import torch.distributed as dist

from tinytron_b200.parallel import parallel_state

from .layout import LayoutIndex, Placement
from .materializers import BridgeContext, RoutedMaterializer
from .planner import LayoutPlanner
from .rules import (EXPERT_SUFFIXES, ParallelSpec, build_tinytron_canonical_layout, build_tinytron_inference_layout,
                    build_tinytron_training_layout)
from .stores import DistributedStateDictStore, StateDictTensorStore

EXPERT_PARAM_SUFFIXES = EXPERT_SUFFIXES


def _sep_size() -> int:
    return parallel_state.get_sep_world_size()


def current_tinytron_parallel_spec(system: str) -> ParallelSpec:
    if dist.is_available() and dist.is_initialized() and parallel_state.model_parallel_is_initialized():
        return ParallelSpec(dp_size=int(parallel_state.get_dp_world_size()),
                            sep_size=int(parallel_state.get_sep_world_size()), system=system)
    return ParallelSpec(dp_size=1, sep_size=1, system=system)


def current_tinytron_placement(layout: LayoutIndex) -> Placement:
    rank = dist.get_rank() if dist.is_available() and dist.is_initialized() else 0
    pls = layout.placements()
    for p in pls:
        if p.rank == rank:
            return p
    if rank == 0 and len(pls) == 1:
        return pls[0]
    raise ValueError(f"layout {layout.name!r} has no placement for global rank {rank}")


def localize_layout(layout: LayoutIndex, placement: Placement) -> LayoutIndex:
    return LayoutIndex.from_shards(name=f"{layout.name}:local:{placement.rank}", shards=layout.local_shards(placement))


def bridge_metadata(*, layout_kind: str, parallel: ParallelSpec, shard_qkv: bool = False,
                    format_version: int = 1) -> dict:
    return {"bridge_format_version": format_version, "layout_kind": layout_kind, "parallel": asdict(parallel),
            "shard_qkv": bool(shard_qkv)}


def _materialize_local(src_sd, src_layout, dst_layout, dst_placement):
    src_store = StateDictTensorStore({src_layout.placements()[0]: src_sd})
    dst_store = StateDictTensorStore()
    plan = LayoutPlanner().plan(src_layout, dst_layout)
    RoutedMaterializer().materialize(plan, BridgeContext(src_store=src_store, dst_store=dst_store))
    return dst_store.state_dict_for(dst_placement)


def _needs_inference_bridge(sd, cfg) -> bool:
    sep = _sep_size()
    if cfg.inference_shard_qkv and sep > 1:
        w = sd.get("blocks.0.attn.q_proj.weight")
        if w is not None and w.size(0) == cfg.hidden_size:
            return True
    if cfg.use_moe and sep > 1:
        w = sd.get("blocks.0.mlp.experts_gate_weights")
        if w is not None and w.size(0) == cfg.num_experts:
            return True
    return False


def _needs_training_bridge(sd, cfg) -> bool:
    if not cfg.use_moe or _sep_size() <= 1:
        return False
    w = sd.get("blocks.0.mlp.experts_gate_weights")
    return w is not None and w.size(0) == cfg.num_experts


def _looks_like_local_training_state_dict(sd, cfg) -> bool:
    sep = _sep_size()
    if not cfg.use_moe or sep <= 1:
        return False
    w = sd.get("blocks.0.mlp.experts_gate_weights")
    return w is not None and w.size(0) == cfg.num_experts // sep


def canonical_state_dict_to_local_inference(state_dict, model_config):
    if not _needs_inference_bridge(state_dict, model_config):
        return state_dict
    dst = build_tinytron_inference_layout(model_config, current_tinytron_parallel_spec("inference"),
                                          shard_qkv=model_config.inference_shard_qkv)
    pl = current_tinytron_placement(dst)
    return _materialize_local(state_dict, build_tinytron_canonical_layout(model_config), localize_layout(dst, pl), pl)


def local_training_state_dict_to_local_inference(state_dict, model_config):
    if not _needs_inference_bridge(state_dict, model_config):
        return state_dict
    src = build_tinytron_training_layout(model_config, current_tinytron_parallel_spec("training"))
    dst = build_tinytron_inference_layout(model_config, current_tinytron_parallel_spec("inference"),
                                          shard_qkv=model_config.inference_shard_qkv)
    dpl = current_tinytron_placement(dst)
    return _materialize_local(state_dict, localize_layout(src, current_tinytron_placement(src)),
                              localize_layout(dst, dpl), dpl)


def state_dict_to_local_inference(state_dict, model_config):
    if _looks_like_local_training_state_dict(state_dict, model_config):
        return local_training_state_dict_to_local_inference(state_dict, model_config)
    return canonical_state_dict_to_local_inference(state_dict, model_config)


def distributed_training_state_dict_to_local_inference(state_dict, model_config, process_group=None,
                                                       use_p2p: bool = True):
    """Live reshard of every rank's training state dict into its inference shard.
    With ``use_p2p`` slices move only between their source and destination ranks, one
    packed transfer per rank pair; otherwise every slice is broadcast (reference semantics)."""
    if not (dist.is_available() and dist.is_initialized()):
        return local_training_state_dict_to_local_inference(state_dict, model_config)
    src = build_tinytron_training_layout(model_config, current_tinytron_parallel_spec("training"))
    dst = build_tinytron_inference_layout(model_config, current_tinytron_parallel_spec("inference"),
                                          shard_qkv=model_config.inference_shard_qkv)
    out: dict[str, torch.Tensor] = {}
    src_store = DistributedStateDictStore(state_dict, process_group=process_group)
    dst_store = DistributedStateDictStore(out, process_group=process_group)
    rank = dist.get_rank()
    ctx = BridgeContext(src_store=src_store, dst_store=dst_store)
    if use_p2p:  # replicated sources share the sending (every rank plans identically)
        plan = LayoutPlanner(balance_sources=True).plan(src, dst)  # one packed transfer per (source, destination) rank pair
        from .materializers import PackedP2PMaterializer

        PackedP2PMaterializer(rank, process_group).materialize(plan, ctx)
        return out
    plan = LayoutPlanner().plan(src, dst)
    from .materializers import DistributedCopyRoute

    RoutedMaterializer(routes=[DistributedCopyRoute(rank)]).materialize(plan, ctx)
    return out


def canonical_state_dict_to_local_training(state_dict, model_config):
    if not _needs_training_bridge(state_dict, model_config):
        return state_dict
    dst = build_tinytron_training_layout(model_config, current_tinytron_parallel_spec("training"))
    pl = current_tinytron_placement(dst)
    return _materialize_local(state_dict, build_tinytron_canonical_layout(model_config), localize_layout(dst, pl), pl)


def _is_expert_param(name: str) -> bool:
    return name.endswith(EXPERT_PARAM_SUFFIXES)
