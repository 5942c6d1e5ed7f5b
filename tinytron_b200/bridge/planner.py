"""Transport-free reshard planner: which slice of which source shard fills which part
of every destination shard (the capability of the reference's
tinytron/bridge/planner.py:16-109; ``LayoutPlanner.plan`` and ``TensorMove`` are its API).

Algorithm (per destination shard, in a fixed order):

* The destination box starts as the only *uncovered* region.  Source shards of the
  same parameter are visited in preference order, and each one contributes its
  intersection with every still-uncovered box; covered pieces are cut out of the
  uncovered set (box difference), so overlapping sources never copy a region twice
  and coverage is exact by construction rather than by counting elements.
* Preference: a source on the destination's own rank first (a local copy, no link
  traffic); then, with ``balance_sources=True``, the source that has been assigned the
  fewest elements so far across the whole plan, so replicated sources (e.g. every DP
  replica of an expert shard) share the outgoing bytes instead of one replica feeding
  every destination — on NVSwitch every pair of GPUs has full bandwidth, so the
  bottleneck is the busiest sender.  Remaining ties go to the lowest slice and rank,
  which keeps the plan deterministic and identical on every rank (and, with balancing
  off, picks the same replicas as the reference planner).
* Anything left uncovered is an error.

``group_by_rank_pair`` buckets a plan by (source rank, destination rank) so a transport
can move all of a pair's slices as one packed transfer.
"""
from __future__ import annotations

from collections import defaultdict
from dataclasses import dataclass

from .layout import LayoutIndex, Placement, ShardSpec, SliceSpec, intersect_slices, local_slices, slice_shape


@dataclass(frozen=True)
class TensorMove:
    """Copy ``global_slices`` of ``param_name`` from ``src_shard`` (at ``src_slices`` in
    its local coordinates) into ``dst_shard`` (at ``dst_slices``)."""

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
        return _volume(self.global_slices)


def _volume(box: tuple[SliceSpec, ...]) -> int:
    n = 1
    for d in slice_shape(box):
        n *= d
    return n


def _subtract(box: tuple[SliceSpec, ...], cut: tuple[SliceSpec, ...]) -> list[tuple[SliceSpec, ...]]:
    """``box`` minus ``cut`` (``cut`` lies inside ``box``) as disjoint boxes: peel the parts
    below and above the cut one dimension at a time."""
    out = []
    rest = list(box)
    for d, ((b0, b1), (c0, c1)) in enumerate(zip(box, cut)):
        if b0 < c0:
            out.append(tuple(rest[:d]) + ((b0, c0),) + tuple(rest[d + 1:]))
        if c1 < b1:
            out.append(tuple(rest[:d]) + ((c1, b1),) + tuple(rest[d + 1:]))
        rest[d] = (c0, c1)
    return out


def _rank(p: Placement) -> int:
    return -1 if p.rank is None else int(p.rank)


class LayoutPlanner:
    """Builds the list of :class:`TensorMove` that turns a source layout into a target one."""

    def __init__(self, balance_sources: bool = False):
        self.balance_sources = bool(balance_sources)

    def plan(self, src: LayoutIndex, dst: LayoutIndex) -> tuple[TensorMove, ...]:
        sources = src.by_param()
        sent: dict[int, int] = defaultdict(int)  # elements each source rank sends to other ranks so far
        moves: list[TensorMove] = []
        for d in sorted(dst.shards, key=_shard_key):
            cands = sources.get(d.param_name)
            if not cands:
                raise KeyError(f"no source shard holds parameter {d.param_name!r}")
            for s in cands:
                if tuple(s.global_shape) != tuple(d.global_shape):
                    raise ValueError(f"shape mismatch for {d.param_name}: source {tuple(s.global_shape)}, "
                                     f"target {tuple(d.global_shape)}")
            uncovered = [tuple(d.global_slices)]
            pieces: list[tuple[tuple[SliceSpec, ...], ShardSpec]] = []
            pool = [s for s in cands if intersect_slices(s.global_slices, d.global_slices) is not None]
            while uncovered and pool:
                s = min(pool, key=lambda c: self._cost(c, d, sent))
                pool.remove(s)
                remaining = []
                for box in uncovered:
                    ov = intersect_slices(s.global_slices, box)
                    if ov is None:
                        remaining.append(box)
                        continue
                    pieces.append((ov, s))
                    if _rank(s.placement) != _rank(d.placement):  # link traffic only
                        sent[_rank(s.placement)] += _volume(ov)
                    remaining.extend(_subtract(box, ov))
                uncovered = remaining
            if uncovered:
                missing = sum(_volume(b) for b in uncovered)
                raise ValueError(f"source layout does not cover target shard {d.param_name!r} at {d.placement}: "
                                 f"{missing} of {_volume(d.global_slices)} elements have no source")
            for ov, s in sorted(pieces, key=lambda item: (item[0], _shard_key(item[1]))):
                moves.append(TensorMove(param_name=d.param_name, src=s.placement, dst=d.placement,
                                        src_slices=local_slices(s.global_slices, ov),
                                        dst_slices=local_slices(d.global_slices, ov), global_slices=ov,
                                        src_shard=s, dst_shard=d))
        return tuple(moves)

    def _cost(self, s: ShardSpec, d: ShardSpec, sent: dict[int, int]) -> tuple:
        remote = not (s.placement.rank is not None and s.placement.rank == d.placement.rank)
        load = sent[_rank(s.placement)] if self.balance_sources else 0
        return (remote, load, _shard_key(s))


def _shard_key(s: ShardSpec) -> tuple:
    return (s.param_name, tuple(s.global_slices), s.placement.sort_key())


def group_by_rank_pair(plan) -> dict[tuple[int, int], list[TensorMove]]:
    """Moves bucketed by (source rank, destination rank), each bucket in plan order."""
    out: dict[tuple[int, int], list[TensorMove]] = defaultdict(list)
    for m in plan:
        out[(_rank(m.src), _rank(m.dst))].append(m)
    return dict(sorted(out.items()))
