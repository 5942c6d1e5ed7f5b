"""Tensor stores the bridge reads from / writes to (reference: tinytron/bridge/stores.py:13-282).

* StateDictTensorStore: placement-keyed in-memory state dicts.
* DistributedStateDictStore: live per-rank state dict; ``read`` is a collective
  (broadcast from the shard's owner), ``send``/``recv`` move one slice between a
  pair of ranks only (used by :class:`~.materializers.P2PCopyRoute`).
* FileTensorStore: one file per (placement, parameter).
* StateDictShardFileStore: read-only per-rank state_dict files (cached).
"""
from __future__ import annotations

import base64
from pathlib import Path
from typing import Callable, Protocol

import torch
import torch.distributed as dist

from .layout import Placement, ShardSpec, SliceSpec, slice_shape, to_torch_slices


class TensorStore(Protocol):
    def read(self, shard: ShardSpec, local_slices: tuple[SliceSpec, ...] | None = None) -> torch.Tensor: ...

    def write(self, shard: ShardSpec, tensor: torch.Tensor, local_slices: tuple[SliceSpec, ...] | None = None) -> None: ...


def _check_shape(t: torch.Tensor, shard: ShardSpec, where: str) -> None:
    if tuple(t.shape) != shard.local_shape:
        raise ValueError(f"stored tensor shape mismatch for {shard.param_name!r} at {where}: "
                         f"got {tuple(t.shape)}, expected {shard.local_shape}")


def _write_into(state: dict, shard: ShardSpec, tensor: torch.Tensor, local_slices, where: str) -> None:
    if local_slices is None:
        if tuple(tensor.shape) != shard.local_shape:
            raise ValueError(f"write shape mismatch for {shard.param_name!r}: got {tuple(tensor.shape)}, "
                             f"expected {shard.local_shape}")
        state[shard.param_name] = tensor.clone()
        return
    cur = state.get(shard.param_name)
    if cur is None:
        cur = torch.empty(shard.local_shape, dtype=tensor.dtype, device=tensor.device)
        state[shard.param_name] = cur
    _check_shape(cur, shard, where)
    cur[to_torch_slices(local_slices)] = tensor


class StateDictTensorStore:
    def __init__(self, state_dicts: dict[Placement, dict[str, torch.Tensor]] | None = None):
        self.state_dicts = state_dicts or {}

    def read(self, shard, local_slices=None):
        try:
            t = self.state_dicts[shard.placement][shard.param_name]
        except KeyError as exc:
            raise KeyError(f"missing tensor {shard.param_name!r} at placement {shard.placement}") from exc
        _check_shape(t, shard, str(shard.placement))
        return t if local_slices is None else t[to_torch_slices(local_slices)]

    def write(self, shard, tensor, local_slices=None):
        _write_into(self.state_dicts.setdefault(shard.placement, {}), shard, tensor, local_slices, str(shard.placement))

    def state_dict_for(self, placement: Placement) -> dict[str, torch.Tensor]:
        return self.state_dicts.setdefault(placement, {})


class DistributedStateDictStore:
    def __init__(self, local_state_dict=None, process_group=None, device=None):
        if not (dist.is_available() and dist.is_initialized()):
            raise RuntimeError("DistributedStateDictStore requires an initialized process group")
        self.local_state_dict = {} if local_state_dict is None else local_state_dict
        self.process_group = process_group
        self.rank = dist.get_rank()
        self.device = torch.device(device) if device is not None else None

    def _like(self, name):
        like = self.local_state_dict.get(name)
        if like is None:
            raise KeyError(f"missing local tensor metadata for {name!r}")
        return like

    def read_local(self, shard, local_slices=None):
        t = self.local_state_dict[shard.param_name]
        _check_shape(t, shard, f"rank {self.rank}")
        return t if local_slices is None else t[to_torch_slices(local_slices)]

    def read(self, shard, local_slices=None):
        """Collective: every rank calls; the owner broadcasts the slice."""
        src = int(shard.placement.rank or 0)
        if self.rank == src:
            t = self.read_local(shard, local_slices).contiguous()
        else:
            shape = slice_shape(local_slices) if local_slices is not None else shard.local_shape
            like = self._like(shard.param_name)
            t = torch.empty(shape, dtype=like.dtype, device=self.device or like.device)
        dist.broadcast(t, src=src, group=self.process_group)
        return t

    def send(self, shard, local_slices, dst_rank: int):
        dist.send(self.read_local(shard, local_slices).contiguous(), dst=dst_rank, group=self.process_group)

    def recv(self, shard, local_slices, src_rank: int, like_name: str | None = None) -> torch.Tensor:
        shape = slice_shape(local_slices) if local_slices is not None else shard.local_shape
        like = self._like(like_name or shard.param_name)
        t = torch.empty(shape, dtype=like.dtype, device=self.device or like.device)
        dist.recv(t, src=src_rank, group=self.process_group)
        return t

    def write(self, shard, tensor, local_slices=None):
        if self.rank != int(shard.placement.rank or 0):
            return
        _write_into(self.local_state_dict, shard, tensor, local_slices, f"rank {self.rank}")

    def state_dict(self):
        return self.local_state_dict


class FileTensorStore:
    def __init__(self, root):
        self.root = Path(root)
        self.root.mkdir(parents=True, exist_ok=True)

    def _path_for(self, shard: ShardSpec) -> Path:
        token = base64.urlsafe_b64encode(repr(shard.placement.sort_key()).encode()).decode().rstrip("=")
        return self.root / f"{token}--{shard.param_name.replace('/', '_').replace('.', '__')}.pt"

    def read(self, shard, local_slices=None):
        t = torch.load(self._path_for(shard), map_location="cpu", weights_only=True)
        _check_shape(t, shard, str(shard.placement))
        return t if local_slices is None else t[to_torch_slices(local_slices)]

    def write(self, shard, tensor, local_slices=None):
        path = self._path_for(shard)
        if local_slices is None:
            if tuple(tensor.shape) != shard.local_shape:
                raise ValueError(f"write shape mismatch for {shard.param_name!r}: got {tuple(tensor.shape)}, "
                                 f"expected {shard.local_shape}")
            torch.save(tensor.detach().cpu(), path)
            return
        cur = torch.load(path, map_location="cpu", weights_only=True) if path.exists() else \
            torch.empty(shard.local_shape, dtype=tensor.dtype)
        cur[to_torch_slices(local_slices)] = tensor.detach().cpu()
        torch.save(cur, path)


class StateDictShardFileStore:
    def __init__(self, path_for_placement: Callable[[Placement], str | Path], map_location="cpu", cache: bool = True):
        self.path_for_placement = path_for_placement
        self.map_location = map_location
        self.cache = cache
        self._cache: dict[Placement, dict[str, torch.Tensor]] = {}

    def _sd(self, placement):
        if self.cache and placement in self._cache:
            return self._cache[placement]
        sd = torch.load(Path(self.path_for_placement(placement)), map_location=self.map_location, weights_only=True)
        if self.cache:
            self._cache[placement] = sd
        return sd

    def read(self, shard, local_slices=None):
        sd = self._sd(shard.placement)
        try:
            t = sd[shard.param_name]
        except KeyError as exc:
            raise KeyError(f"missing tensor {shard.param_name!r} at placement {shard.placement}") from exc
        _check_shape(t, shard, str(shard.placement))
        return t if local_slices is None else t[to_torch_slices(local_slices)]

    def write(self, shard, tensor, local_slices=None):
        raise NotImplementedError("StateDictShardFileStore is read-only")
