"""Transport-free reshard planner (reference: tinytron/bridge/planner.py:16-109).

For every destination shard, intersect it with each source shard of the same
parameter; when several sources (replicas) cover the same region, one is chosen,
preferring a source on the destination's own rank (a local copy).  The chosen
pieces must cover the destination exactly, else the plan is rejected.
"""
from __future__ import annotations

from dataclasses import dataclass

from .layout import LayoutIndex, Placement, ShardSpec, SliceSpec, intersect_slices, local_slices, slice_shape


@dataclass(frozen=True)
class TensorMove:
    param_name: str
    src: Placement
    dst: Placement
    src_slices: tuple[SliceSpec, ...]
    dst_slices: tuple[SliceSpec, ...]
    global_slices: tuple[SliceSpec, ...]
    src_shard: ShardSpec
    dst_shard: ShardSpec
    op: str = "copy"

    @property
    def numel(self) -> int:
        n = 1
        for d in slice_shape(self.global_slices):
            n *= d
        return n


def _numel(shape) -> int:
    n = 1
    for d in shape:
        n *= d
    return n


class LayoutPlanner:
    def plan(self, src: LayoutIndex, dst: LayoutIndex) -> tuple[TensorMove, ...]:
        by_param = src.by_param()
        moves: list[TensorMove] = []
        for d in sorted(dst.shards, key=self._key):
            cands = by_param.get(d.param_name)
            if not cands:
                raise KeyError(f"source layout has no shards for parameter {d.param_name!r}")
            chosen: dict[tuple[SliceSpec, ...], ShardSpec] = {}
            for s in sorted(cands, key=self._key):
                if s.global_shape != d.global_shape:
                    raise ValueError(f"shape mismatch for {d.param_name}: source {s.global_shape}, "
                                     f"target {d.global_shape}")
                ov = intersect_slices(s.global_slices, d.global_slices)
                if ov is None:
                    continue
                cur = chosen.get(ov)
                if cur is None or self._prefer_source(s, cur, d):
                    chosen[ov] = s
            self._validate_coverage(d, chosen)
            for ov, s in sorted(chosen.items()):
                moves.append(TensorMove(param_name=d.param_name, src=s.placement, dst=d.placement,
                                        src_slices=local_slices(s.global_slices, ov),
                                        dst_slices=local_slices(d.global_slices, ov), global_slices=ov,
                                        src_shard=s, dst_shard=d))
        return tuple(moves)

    def _validate_coverage(self, dst: ShardSpec, chosen) -> None:
        covered = sum(_numel(slice_shape(ov)) for ov in chosen)
        expected = _numel(dst.local_shape)
        if covered != expected:
            raise ValueError(f"source layout does not cover target shard {dst.param_name!r} at {dst.placement}: "
                             f"covered {covered} elements, expected {expected}")

    def _key(self, shard: ShardSpec) -> tuple:
        return (shard.param_name, shard.global_slices, shard.placement.sort_key())

    def _prefer_source(self, candidate: ShardSpec, current: ShardSpec, dst: ShardSpec) -> bool:
        return candidate.placement.rank == dst.placement.rank and current.placement.rank != dst.placement.rank
