"""Plan execution (reference: tinytron/bridge/materializers.py:12-76).

Routes: LocalCopyRoute (read + write in-process), DistributedCopyRoute (reference
semantics: a broadcast per move), and P2PCopyRoute (only the source and
destination ranks of a move participate: local copy when they coincide, else one
send/recv pair; all ranks walk the plan in the same order so pairs match).

PackedP2PMaterializer (used for live training -> inference resharding) sends each
(source rank, destination rank) pair's slices as ONE packed buffer, and posts all of
this rank's sends and receives as one batch, so a reshard costs one transfer per pair
instead of one per tensor slice.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import TYPE_CHECKING, Protocol

from .layout import slice_shape
from .planner import TensorMove, group_by_rank_pair

if TYPE_CHECKING:
    from .stores import TensorStore


@dataclass
class BridgeContext:
    src_store: "TensorStore"
    dst_store: "TensorStore"


class TensorRoute(Protocol):
    def can_materialize(self, move: TensorMove, context: BridgeContext) -> bool: ...

    def materialize(self, move: TensorMove, context: BridgeContext) -> None: ...


class LocalCopyRoute:
    def can_materialize(self, move, context) -> bool:
        return True

    def materialize(self, move, context) -> None:
        context.dst_store.write(move.dst_shard, context.src_store.read(move.src_shard, move.src_slices),
                                move.dst_slices)


class DistributedCopyRoute:
    def __init__(self, rank: int):
        self.rank = int(rank)

    def can_materialize(self, move, context) -> bool:
        return True

    def materialize(self, move, context) -> None:
        src, dst = int(move.src.rank or 0), int(move.dst.rank or 0)
        if src == dst:
            if self.rank == dst:
                read = getattr(context.src_store, "read_local", context.src_store.read)
                context.dst_store.write(move.dst_shard, read(move.src_shard, move.src_slices), move.dst_slices)
            return
        t = context.src_store.read(move.src_shard, move.src_slices)
        if self.rank == dst:
            context.dst_store.write(move.dst_shard, t, move.dst_slices)


class P2PCopyRoute:
    def __init__(self, rank: int):
        self.rank = int(rank)

    def can_materialize(self, move, context) -> bool:
        return hasattr(context.src_store, "send") and hasattr(context.src_store, "recv")

    def materialize(self, move, context) -> None:
        src, dst = int(move.src.rank or 0), int(move.dst.rank or 0)
        if self.rank == src and self.rank == dst:
            context.dst_store.write(move.dst_shard, context.src_store.read_local(move.src_shard, move.src_slices),
                                    move.dst_slices)
        elif self.rank == src:
            context.src_store.send(move.src_shard, move.src_slices, dst)
        elif self.rank == dst:
            t = context.src_store.recv(move.src_shard, move.src_slices, src)
            context.dst_store.write(move.dst_shard, t, move.dst_slices)


class RoutedMaterializer:
    def __init__(self, routes=None):
        self.routes = routes or [LocalCopyRoute()]

    def materialize(self, plan, context: BridgeContext) -> None:
        for move in plan:
            self._route_for(move, context).materialize(move, context)

    def _route_for(self, move, context):
        for r in self.routes:
            if r.can_materialize(move, context):
                return r
        raise RuntimeError(f"no bridge route can materialize move: {move}")


class PackedP2PMaterializer:
    """Executes a plan over a process group with one packed transfer per rank pair.

    Within a pair, moves are packed in plan order and split by dtype (sender and
    receiver derive the same grouping from the plan and the parameter dtypes).  Copies
    whose source and destination are this rank never leave the device."""

    def __init__(self, rank: int, process_group=None):
        self.rank = int(rank)
        self.process_group = process_group

    def materialize(self, plan, context: BridgeContext) -> None:
        import torch
        import torch.distributed as dist

        src_store, dst_store = context.src_store, context.dst_store
        ops, inbound = [], []
        for (s, d), moves in group_by_rank_pair(plan).items():
            if self.rank not in (s, d):
                continue
            if s == d:
                for m in moves:
                    dst_store.write(m.dst_shard, src_store.read_local(m.src_shard, m.src_slices), m.dst_slices)
                continue
            by_dtype: dict[str, list[TensorMove]] = {}
            for m in moves:
                by_dtype.setdefault(str(src_store._like(m.param_name).dtype), []).append(m)
            for key in sorted(by_dtype):
                group = by_dtype[key]
                if self.rank == s:
                    packed = torch.cat([src_store.read_local(m.src_shard, m.src_slices).reshape(-1) for m in group])
                    ops.append(dist.P2POp(dist.isend, packed, d, group=self.process_group))
                else:
                    like = src_store._like(group[0].param_name)
                    buf = torch.empty(sum(m.numel for m in group), dtype=like.dtype,
                                      device=src_store.device or like.device)
                    ops.append(dist.P2POp(dist.irecv, buf, s, group=self.process_group))
                    inbound.append((buf, group))
        if ops:
            for req in dist.batch_isend_irecv(ops):
                req.wait()
        for buf, group in inbound:
            off = 0
            for m in group:
                n = m.numel
                dst_store.write(m.dst_shard, buf[off:off + n].view(slice_shape(m.global_slices)), m.dst_slices)
                off += n
