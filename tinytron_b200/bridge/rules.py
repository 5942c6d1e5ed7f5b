"""Tinytron layouts (reference: tinytron/bridge/rules.py:10-241).

``ParallelSpec(dp, sep)`` enumerates placements with coordinates (dp, sep, ep=sep),
global rank = dp*sep_size + sep.  Layouts:
  * canonical: one placement, every tensor full;
  * training: expert tensors dim-0 sharded by SEP rank, everything else replicated;
  * inference: as training, plus q/k/v dim-0 sharded by SEP rank when shard_qkv.
``_global_param_shapes`` is the checkpoint key schema.
"""
from __future__ import annotations

from dataclasses import dataclass

from .layout import LayoutIndex, Placement, RankCoord, ShardSpec, SliceSpec, full_slice

EXPERT_SUFFIXES = (".mlp.experts_gate_weights", ".mlp.experts_up_weights", ".mlp.experts_down_weights")
QKV_SUFFIXES = (".attn.q_proj.weight", ".attn.k_proj.weight", ".attn.v_proj.weight")


@dataclass(frozen=True)
class ParallelSpec:
    dp_size: int = 1
    sep_size: int = 1
    system: str = "training"
    group_id: str | None = None

    def placements(self) -> tuple[Placement, ...]:
        return tuple(
            Placement(system=self.system, rank=d * self.sep_size + s,
                      coord=RankCoord.from_axes(dp=d, sep=s, ep=s), group_id=self.group_id)
            for d in range(self.dp_size) for s in range(self.sep_size))


def _global_param_shapes(model_config) -> tuple[tuple[str, tuple[int, ...]], ...]:
    c = model_config
    H = c.hidden_size
    hd = H // c.num_attention_heads
    q_out, kv_out = c.num_attention_heads * hd, c.num_key_value_heads * hd
    shapes: list[tuple[str, tuple[int, ...]]] = [("wte.weight", (c.vocab_size, H))]
    for l in range(c.num_layer):
        p = f"blocks.{l}"
        shapes += [(f"{p}.ln_1.weight", (H,)), (f"{p}.attn.q_proj.weight", (q_out, H)),
                   (f"{p}.attn.k_proj.weight", (kv_out, H)), (f"{p}.attn.v_proj.weight", (kv_out, H)),
                   (f"{p}.attn.c_proj.weight", (H, H)), (f"{p}.ln_2.weight", (H,))]
        if c.use_moe:
            I, E = c.moe_intermediate_size, c.num_experts
            shapes += [(f"{p}.mlp.router.weight", (E, H)), (f"{p}.mlp.experts_gate_weights", (E, I, H)),
                       (f"{p}.mlp.experts_up_weights", (E, I, H)), (f"{p}.mlp.experts_down_weights", (E, H, I))]
        else:
            I = c.intermediate_size
            shapes += [(f"{p}.mlp.gate_proj.weight", (I, H)), (f"{p}.mlp.up_proj.weight", (I, H)),
                       (f"{p}.mlp.down_proj.weight", (H, I))]
    shapes += [("lnf.weight", (H,)), ("lm_head.weight", (c.vocab_size, H))]
    return tuple(shapes)


def _is_expert_param(name: str) -> bool:
    return name.endswith(EXPERT_SUFFIXES)


def _is_qkv_param(name: str) -> bool:
    return name.endswith(QKV_SUFFIXES)


def _axis(p: Placement, axis: str) -> int:
    if p.coord is None:
        raise ValueError(f"placement {p} has no rank coordinate")
    v = p.coord.get(axis)
    if v is None:
        raise ValueError(f"placement {p} has no {axis!r} coordinate")
    return v


def _dim0_shard(name, shape, placement, rank, world, tag) -> ShardSpec:
    if shape[0] % world:
        raise ValueError(f"{name} dim0={shape[0]} must be divisible by world_size={world}")
    chunk = shape[0] // world
    sl: list[SliceSpec] = list(full_slice(shape))
    sl[0] = (rank * chunk, (rank + 1) * chunk)
    return ShardSpec(param_name=name, global_shape=shape, global_slices=tuple(sl), placement=placement,
                     axis_tags=(tag,))


def build_tinytron_canonical_layout(model_config, system: str = "canonical") -> LayoutIndex:
    pl = Placement(system=system, rank=0, coord=RankCoord.from_axes(replica=0))
    return LayoutIndex.from_shards("tinytron-canonical",
                                   [ShardSpec.replicated(n, s, pl) for n, s in _global_param_shapes(model_config)])


def _build(model_config, parallel: ParallelSpec, name: str, shard_qkv: bool) -> LayoutIndex:
    pls = parallel.placements()
    shards: list[ShardSpec] = []
    for n, s in _global_param_shapes(model_config):
        for p in pls:
            if shard_qkv and _is_qkv_param(n):
                shards.append(_dim0_shard(n, s, p, _axis(p, "sep"), parallel.sep_size, "qkv_head"))
            elif _is_expert_param(n):
                shards.append(_dim0_shard(n, s, p, _axis(p, "sep"), parallel.sep_size, "expert"))
            else:
                shards.append(ShardSpec.replicated(n, s, p, replica_group=f"{parallel.system}:{n}"))
    return LayoutIndex.from_shards(name, shards)


def build_tinytron_training_layout(model_config, parallel: ParallelSpec) -> LayoutIndex:
    return _build(model_config, parallel, "tinytron-training", shard_qkv=False)


def build_tinytron_inference_layout(model_config, parallel: ParallelSpec, shard_qkv: bool = False) -> LayoutIndex:
    return _build(model_config, parallel, "tinytron-inference", shard_qkv=shard_qkv)
