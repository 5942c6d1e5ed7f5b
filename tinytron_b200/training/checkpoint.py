"""Checkpoint file policy (reference: tinytron/training/checkpoint.py:27-133).

Files per save, prefix ``<log_dir>/<step:05d>`` (identical names and meta keys to
the reference, so checkpoints interoperate):
  ``_model_rank{r:05d}.pt`` per-rank fp32 state dict (experts: local shard),
  ``_model.pt`` rank-0 legacy copy, ``_meta.pt``, ``_opt/`` (DCP, key
  ``optimizer/rank{r}``), ``_rng/rank{r}.pt``.
Extras: each model shard gets a ``.crc32`` sidecar checked on load (a corrupt
shard raises instead of loading garbage).  Resharding across SEP sizes goes
through the bridge planner.
"""
from __future__ import annotations

import glob
import os
import zlib
from dataclasses import asdict

import torch
import torch.distributed as dist

from tinytron_b200.bridge import (BridgeContext, LayoutPlanner, ParallelSpec, RoutedMaterializer,
                                  StateDictShardFileStore, StateDictTensorStore, bridge_metadata,
                                  build_tinytron_canonical_layout, build_tinytron_training_layout,
                                  canonical_state_dict_to_local_training, current_tinytron_parallel_spec,
                                  current_tinytron_placement, localize_layout)


class CheckpointCorruptError(RuntimeError):
    pass


def checkpoint_prefix_from_model_path(model_path: str) -> str:
    if model_path.endswith("_model_canonical.pt"):
        return model_path[: -len("_model_canonical.pt")]
    if model_path.endswith("_model.pt"):
        return model_path[: -len("_model.pt")]
    if "_model_rank" in model_path and model_path.endswith(".pt"):
        return model_path.rsplit("_model_rank", 1)[0]
    raise ValueError(f"Cannot infer checkpoint prefix from model path: {model_path}")


def checkpoint_meta_path(prefix: str) -> str:
    return f"{prefix}_meta.pt"


def checkpoint_model_path(prefix: str) -> str:
    return f"{prefix}_model.pt"


def checkpoint_model_shard_path(prefix: str, rank: int) -> str:
    return f"{prefix}_model_rank{rank:05d}.pt"


def find_latest_checkpoint_prefix(checkpoint_dir: str) -> str | None:
    found = sorted(glob.glob(os.path.join(checkpoint_dir, "*_model.pt")))
    return checkpoint_prefix_from_model_path(found[-1]) if found else None


def model_layout_metadata() -> dict:
    return bridge_metadata(layout_kind="training", parallel=current_tinytron_parallel_spec(system="training"),
                           shard_qkv=False)


def training_layout_matches_current(meta: dict) -> bool:
    layout = meta.get("model_layout")
    if layout is None:
        return True
    if layout.get("layout_kind") != "training":
        return False
    return layout.get("parallel") == asdict(current_tinytron_parallel_spec(system="training"))


# ------------------------------------------------------------------ integrity sidecars
def _crc32(path: str) -> int:
    crc = 0
    with open(path, "rb") as f:
        for chunk in iter(lambda: f.read(1 << 24), b""):
            crc = zlib.crc32(chunk, crc)
    return crc & 0xFFFFFFFF


def _write_crc(path: str) -> None:
    with open(path + ".crc32", "w") as f:
        f.write(f"{_crc32(path):08x}\n")


def verify_checksum(path: str) -> None:
    side = path + ".crc32"
    if not os.path.exists(side):
        return
    want = open(side).read().strip()
    got = f"{_crc32(path):08x}"
    if want != got:
        raise CheckpointCorruptError(f"checksum mismatch for {path}: expected {want}, got {got}")


def write_checksums(prefix: str) -> None:
    p = checkpoint_model_path(prefix)
    if os.path.exists(p):
        _write_crc(p)


def _load(path: str):
    verify_checksum(path)
    return torch.load(path, map_location="cpu", weights_only=True)


def save_local_model_shard(model, prefix: str, rank: int) -> None:
    path = checkpoint_model_shard_path(prefix, rank)
    torch.save(model.state_dict(), path)
    _write_crc(path)


def save_rank0_legacy_model(model, prefix: str) -> None:
    torch.save(model.state_dict(), checkpoint_model_path(prefix))


# ------------------------------------------------------------------ optimizer (DCP)
def save_optimizer_state(optimizer, prefix: str, rank: int) -> None:
    sd = {f"optimizer/rank{rank}": optimizer.state_dict()}
    if dist.is_initialized():
        from torch.distributed.checkpoint import FileSystemWriter, state_dict_saver

        state_dict_saver.save(state_dict=sd, storage_writer=FileSystemWriter(f"{prefix}_opt"))
    else:
        os.makedirs(f"{prefix}_opt", exist_ok=True)
        torch.save(sd, os.path.join(f"{prefix}_opt", f"rank{rank}.pt"))


def load_optimizer_state(optimizer, prefix: str, rank: int) -> None:
    key = f"optimizer/rank{rank}"
    plain = os.path.join(f"{prefix}_opt", f"rank{rank}.pt")
    if os.path.exists(plain):
        optimizer.load_state_dict(torch.load(plain, map_location="cpu", weights_only=False)[key])
        return
    from torch.distributed.checkpoint import FileSystemReader, state_dict_loader

    holder = {key: optimizer.state_dict()}
    state_dict_loader.load(state_dict=holder, storage_reader=FileSystemReader(f"{prefix}_opt"))
    optimizer.load_state_dict(holder[key])


# ------------------------------------------------------------------ model load / reshard
def load_model_state_dict_for_training(checkpoint_prefix: str, model_config, rank: int, meta: dict):
    own = checkpoint_model_shard_path(checkpoint_prefix, rank)
    if os.path.exists(own) and training_layout_matches_current(meta):
        return _load(own)
    if _has_sharded_model_checkpoint(checkpoint_prefix, meta):
        return _reshard_model_state_dict_from_files(checkpoint_prefix, model_config, meta)
    path = checkpoint_model_path(checkpoint_prefix)
    canonical = f"{checkpoint_prefix}_model_canonical.pt"
    if not os.path.exists(path) and os.path.exists(canonical):
        path = canonical
    sd = _load(path)
    if path.endswith("_model_canonical.pt"):
        return canonical_state_dict_to_local_training(sd, model_config)
    return sd


def _has_sharded_model_checkpoint(prefix: str, meta: dict) -> bool:
    return bool(meta.get("model_sharded")) and os.path.exists(checkpoint_model_shard_path(prefix, 0))


class _VerifiedShardStore(StateDictShardFileStore):
    def _sd(self, placement):
        if self.cache and placement in self._cache:
            return self._cache[placement]
        verify_checksum(str(self.path_for_placement(placement)))
        return super()._sd(placement)


def _reshard_model_state_dict_from_files(prefix: str, model_config, meta: dict):
    src = _source_layout_from_meta(meta, model_config)
    dst = build_tinytron_training_layout(model_config, current_tinytron_parallel_spec(system="training"))
    pl = current_tinytron_placement(dst)
    store = _VerifiedShardStore(lambda p: checkpoint_model_shard_path(prefix, int(p.rank or 0)))
    out = StateDictTensorStore()
    plan = LayoutPlanner().plan(src, localize_layout(dst, pl))
    RoutedMaterializer().materialize(plan, BridgeContext(src_store=store, dst_store=out))
    return out.state_dict_for(pl)


def _source_layout_from_meta(meta: dict, model_config):
    layout = meta.get("model_layout") or {}
    kind = layout.get("layout_kind", "training")
    parallel = ParallelSpec(**layout.get("parallel", asdict(current_tinytron_parallel_spec(system="training"))))
    if kind == "training":
        return build_tinytron_training_layout(model_config=model_config, parallel=parallel)
    if kind == "canonical":
        return build_tinytron_canonical_layout(model_config=model_config)
    raise ValueError(f"Unsupported checkpoint model layout kind: {kind}")
