"""Packed scalar all-reduce: every small statistic of a training micro-step crosses the
ranks in ONE collective.

The reference issues a separate NCCL all-reduce for each of them: the valid-token
counts over SP and DP (tinytron/training/trainer.py:359-361), the cross-entropy
statistics over SP (model/modules/loss.py:34,40) and two per MoE layer for the
load-balancing statistics (loss.py:72-78), i.e. 35 collectives per micro-step for a
16-layer MoE.  Here the model gathers all of them into one fp32 vector at the end of
its forward and reduces it once; per-rank quantities that are needed as sums over a
SUB-group (the SP/EP group) travel in one slot per rank, so a single reduction over
the DP x SP group yields every group's sum.

On CUDA inside one node the reduction runs on a small symmetric heap with the
graph-safe two-kernel all-reduce (device-side epochs; peer loads over NVLink);
otherwise (CPU/gloo, several nodes, ``--comm_impl nccl``) it is one ``dist.all_reduce``.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

_MAX_FLOATS = 16384
_REDUCERS: dict = {}


class _HeapScalarReducer:
    def __init__(self, group, device):
        from .symm import SymmetricHeap

        self.heap = SymmetricHeap.create(2 * _MAX_FLOATS * 4 + 4096, group, device)
        self.slots, self.slot_bytes = self.heap.replay_slots(_MAX_FLOATS * 4)

    def __call__(self, vec: torch.Tensor) -> torch.Tensor:
        out = torch.empty_like(vec)
        self.heap.replay_publish(self.slots, self.slot_bytes, vec)
        self.heap.replay_reduce(self.slots, self.slot_bytes, out)
        return out

    def close(self):
        self.heap.close()


def _reducer(group, device):
    key = id(group)
    if key not in _REDUCERS:
        r = None
        from . import parallel_state
        from .symm import same_host

        if (device.type == "cuda" and parallel_state.native_comm_enabled() and dist.get_world_size(group) <= 8
                and same_host(group)):
            r = _HeapScalarReducer(group, device)
        _REDUCERS[key] = r
    return _REDUCERS[key]


def all_reduce_scalars(vec: torch.Tensor, group) -> torch.Tensor:
    """Sum of a small fp32 vector over ``group`` (a new tensor; ``vec`` is not modified).
    Collective: every rank of the group calls it with the same length."""
    if group is None or not dist.is_initialized() or dist.get_world_size(group) == 1:
        return vec.clone()
    n = vec.numel()
    if n > _MAX_FLOATS:
        raise ValueError(f"packed scalar all-reduce holds at most {_MAX_FLOATS} floats, got {n}")
    padded = torch.zeros((n + 3) // 4 * 4, dtype=torch.float32, device=vec.device)
    padded[:n] = vec.reshape(-1).float()
    red = _reducer(group, vec.device)
    if red is not None:
        return red(padded)[:n].view_as(vec)
    dist.all_reduce(padded, op=dist.ReduceOp.SUM, group=group)
    return padded[:n].view_as(vec)


def release_scalar_reducers() -> None:
    for r in _REDUCERS.values():
        if r is not None:
            r.close()
    _REDUCERS.clear()


def rank_slot_vector(value: torch.Tensor, world_rank: int, world: int) -> torch.Tensor:
    """A [world] fp32 vector holding ``value`` at this rank's slot and zeros elsewhere."""
    v = torch.zeros(world, dtype=torch.float32, device=value.device)
    v[world_rank] = value.float()
    return v
