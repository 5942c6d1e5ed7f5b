"""Plan execution (reference: tinytron/bridge/materializers.py:12-76).

Routes: LocalCopyRoute (read + write in-process), DistributedCopyRoute (reference
semantics: a broadcast per move), and P2PCopyRoute (only the source and
destination ranks of a move participate: local copy when they coincide, else one
send/recv pair; all ranks walk the plan in the same order so pairs match).
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import TYPE_CHECKING, Protocol

from .planner import TensorMove

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
