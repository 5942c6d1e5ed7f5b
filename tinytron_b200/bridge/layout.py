"""Layout algebra for the checkpoint / weight-sync bridge
(reference: tinytron/bridge/layout.py:8-163).

A parameter's placement in some "world" (training ranks, inference ranks, a file,
a canonical full copy) is a :class:`ShardSpec`: the global shape, the half-open
global slice this shard holds, and a :class:`Placement`.  A :class:`LayoutIndex` is
the set of shards of every parameter in a world.  Slices are tuples of
(start, stop) per dimension.
"""
from __future__ import annotations

from collections import defaultdict
from dataclasses import dataclass, field
from typing import Iterable

SliceSpec = tuple[int, int]


@dataclass(frozen=True)
class RankCoord:
    """Named logical coordinates (e.g. dp=0, sep=1, ep=1), order-independent."""

    axes: tuple[tuple[str, int], ...] = ()

    @classmethod
    def from_axes(cls, **axes: int) -> "RankCoord":
        return cls(tuple(sorted((str(k), int(v)) for k, v in axes.items())))

    def get(self, axis: str, default: int | None = None) -> int | None:
        for k, v in self.axes:
            if k == axis:
                return v
        return default


@dataclass(frozen=True)
class Placement:
    """Where a shard lives.  ``system`` names the world; the other fields are
    descriptive metadata that routes may use."""

    system: str
    rank: int | None = None
    coord: RankCoord | None = None
    group_id: str | None = None
    address: str | None = None
    metadata: tuple[tuple[str, str], ...] = ()

    def sort_key(self) -> tuple:
        return (self.system, -1 if self.rank is None else self.rank, self.group_id or "", self.address or "",
                self.coord.axes if self.coord is not None else (), self.metadata)


def full_slice(shape: tuple[int, ...]) -> tuple[SliceSpec, ...]:
    return tuple((0, int(d)) for d in shape)


def slice_shape(slices: tuple[SliceSpec, ...]) -> tuple[int, ...]:
    return tuple(b - a for a, b in slices)


def intersect_slices(left: tuple[SliceSpec, ...], right: tuple[SliceSpec, ...]) -> tuple[SliceSpec, ...] | None:
    if len(left) != len(right):
        raise ValueError(f"slice rank mismatch: {len(left)} vs {len(right)}")
    out = []
    for (a0, a1), (b0, b1) in zip(left, right):
        lo, hi = max(a0, b0), min(a1, b1)
        if lo >= hi:
            return None
        out.append((lo, hi))
    return tuple(out)


def to_torch_slices(slices: tuple[SliceSpec, ...]) -> tuple[slice, ...]:
    return tuple(slice(a, b) for a, b in slices)


def local_slices(shard_slices: tuple[SliceSpec, ...], global_slices: tuple[SliceSpec, ...]) -> tuple[SliceSpec, ...]:
    """Express a global sub-slice in the shard's local coordinates."""
    if len(shard_slices) != len(global_slices):
        raise ValueError(f"slice rank mismatch: {len(shard_slices)} vs {len(global_slices)}")
    out = []
    for (s0, s1), (g0, g1) in zip(shard_slices, global_slices):
        if g0 < s0 or g1 > s1:
            raise ValueError(f"global slice {(g0, g1)} is outside shard slice {(s0, s1)}")
        out.append((g0 - s0, g1 - s0))
    return tuple(out)


@dataclass(frozen=True)
class ShardSpec:
    param_name: str
    global_shape: tuple[int, ...]
    global_slices: tuple[SliceSpec, ...]
    placement: Placement
    axis_tags: tuple[str, ...] = ()
    replica_group: str | None = None
    metadata: tuple[tuple[str, str], ...] = ()

    @property
    def local_shape(self) -> tuple[int, ...]:
        return slice_shape(self.global_slices)

    @classmethod
    def replicated(cls, param_name: str, global_shape: tuple[int, ...], placement: Placement,
                   replica_group: str | None = None) -> "ShardSpec":
        shape = tuple(int(d) for d in global_shape)
        return cls(param_name=param_name, global_shape=shape, global_slices=full_slice(shape), placement=placement,
                   replica_group=replica_group)


@dataclass(frozen=True)
class LayoutIndex:
    name: str
    shards: tuple[ShardSpec, ...] = field(default_factory=tuple)

    def __post_init__(self) -> None:
        object.__setattr__(self, "shards", tuple(self.shards))

    @classmethod
    def from_shards(cls, name: str, shards: Iterable[ShardSpec]) -> "LayoutIndex":
        return cls(name=name, shards=tuple(shards))

    @property
    def param_names(self) -> tuple[str, ...]:
        return tuple(sorted({s.param_name for s in self.shards}))

    def shards_for(self, param_name: str) -> tuple[ShardSpec, ...]:
        return tuple(s for s in self.shards if s.param_name == param_name)

    def local_shards(self, placement: Placement) -> tuple[ShardSpec, ...]:
        return tuple(s for s in self.shards if s.placement == placement)

    def placements(self) -> tuple[Placement, ...]:
        return tuple(sorted({s.placement for s in self.shards}, key=lambda p: p.sort_key()))

    def by_param(self) -> dict[str, tuple[ShardSpec, ...]]:
        grouped: dict[str, list[ShardSpec]] = defaultdict(list)
        for s in self.shards:
            grouped[s.param_name].append(s)
        return {k: tuple(sorted(v, key=lambda s: s.placement.sort_key())) for k, v in grouped.items()}
