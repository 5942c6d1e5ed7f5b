"""Streaming pretraining data: fixed-length samples read straight from token shards on disk,
split across data-parallel ranks, with a resumable position (the capability of the
reference's example entry point, scripts/example/pretrain.py:76-294, which relies on an
external Streaming-Dataloader package).

On-disk format (written by :func:`write_token_shards`, or by any tokenizer pipeline):

    <dir>/meta.json       {"dtype": "uint16" | "uint32", "chunks": [{"file": ..., "tokens": n}, ...]}
    <dir>/chunk_00000.bin raw little-endian token ids, concatenated documents

Every shard is memory-mapped (numpy), so a worker touches only the pages of the samples
it reads.  Sample i covers tokens [i * seq_len, i * seq_len + seq_len + 1) of the
concatenated stream (inputs and next-token labels); rank r of a DP group of size W reads
samples r, r + W, r + 2W, ... in order, optionally in a seeded per-epoch permutation.
The position is "globally consumed samples": ``global_skip`` samples are skipped at the
start (resume), and :class:`StreamingTrainer` stores the next value in its checkpoints.
"""
from __future__ import annotations

import json
import os

import numpy as np
import torch
from torch.utils.data import DataLoader, IterableDataset, get_worker_info

from .trainer import Trainer

_DTYPES = {"uint16": np.uint16, "uint32": np.uint32, "int32": np.int32}


def write_token_shards(out_dir: str, tokens: np.ndarray, tokens_per_chunk: int = 1 << 24,
                       dtype: str = "uint16") -> None:
    """Write a 1-D token array as shards + meta.json (the format :class:`TokenShardDataset` reads)."""
    os.makedirs(out_dir, exist_ok=True)
    arr = np.asarray(tokens).astype(_DTYPES[dtype])
    chunks = []
    for i, s in enumerate(range(0, arr.size, tokens_per_chunk)):
        name = f"chunk_{i:05d}.bin"
        part = arr[s:s + tokens_per_chunk]
        part.tofile(os.path.join(out_dir, name))
        chunks.append({"file": name, "tokens": int(part.size)})
    with open(os.path.join(out_dir, "meta.json"), "w") as f:
        json.dump({"dtype": dtype, "chunks": chunks}, f)


class TokenShardDataset(IterableDataset):
    def __init__(self, data_dir: str, seq_len: int, dp_rank: int = 0, dp_world_size: int = 1, shuffle: bool = False,
                 seed: int = 0, global_skip: int = 0, strict: bool = True):
        with open(os.path.join(data_dir, "meta.json")) as f:
            meta = json.load(f)
        self.data_dir = data_dir
        self.dtype = _DTYPES[meta["dtype"]]
        self.chunks = [(c["file"], int(c["tokens"])) for c in meta["chunks"]]
        self.starts = np.cumsum([0] + [n for _, n in self.chunks])
        self.total_tokens = int(self.starts[-1])
        self.seq_len = int(seq_len)
        self.total_samples = max(0, (self.total_tokens - 1) // self.seq_len)
        self.dp_rank, self.dp_world_size = int(dp_rank), int(dp_world_size)
        self.shuffle, self.seed = bool(shuffle), int(seed)
        self.global_skip = int(global_skip)
        self.epoch = 0
        self._maps = None
        if strict and self.total_samples < self.dp_world_size:
            raise ValueError(f"{self.total_samples} samples cannot feed {self.dp_world_size} data-parallel ranks")

    def set_epoch(self, epoch: int) -> None:
        self.epoch = int(epoch)

    def _mmaps(self):
        if self._maps is None:
            self._maps = [np.memmap(os.path.join(self.data_dir, f), dtype=self.dtype, mode="r", shape=(n,))
                          for f, n in self.chunks]
        return self._maps

    def _tokens(self, start: int, count: int) -> np.ndarray:
        """Tokens [start, start + count) of the concatenated stream (may span shards)."""
        maps, out, pos = self._mmaps(), [], start
        while count > 0:
            c = int(np.searchsorted(self.starts, pos, side="right") - 1)
            off = pos - int(self.starts[c])
            take = min(count, self.chunks[c][1] - off)
            out.append(np.asarray(maps[c][off:off + take]))
            pos += take
            count -= take
        return np.concatenate(out) if len(out) > 1 else out[0]

    def _order(self) -> np.ndarray:
        if not self.shuffle:
            return np.arange(self.total_samples)
        return np.random.default_rng(self.seed + self.epoch).permutation(self.total_samples)

    def __iter__(self):
        order = self._order()
        first = self.global_skip + self.dp_rank  # global sample index of this rank's first sample
        idx = np.arange(first, self.total_samples, self.dp_world_size)
        info = get_worker_info()
        if info is not None:  # DataLoader workers split this rank's samples round-robin
            idx = idx[info.id::info.num_workers]
        for i in idx:
            s = int(order[i]) * self.seq_len
            data = torch.from_numpy(self._tokens(s, self.seq_len + 1).astype(np.int64))
            yield {"input_ids": data[:-1], "labels": data[1:]}


class StreamingTrainer(Trainer):
    """Trainer reading :class:`TokenShardDataset` (``--dataset_path`` is the shard
    directory); checkpoints carry the dataset position, and resuming continues with the
    next unconsumed sample even across epochs."""

    streaming_shuffle = False

    def _global_samples_per_step(self) -> int:
        return self.training_info["grad_accum_steps"] * self.config.train.batch_size * self.dp_world_size

    def _init_dataset(self, config):
        if config.data.use_mock_data:
            return super()._init_dataset(config)
        self.train_dataset = TokenShardDataset(config.data.dataset_path, config.train.seq_len, self.dp_rank,
                                               self.dp_world_size, shuffle=self.streaming_shuffle,
                                               seed=config.seed.seed)
        self.val_dataset = self.val_loader = self.train_sampler = self.val_sampler = None
        self.train_loader = DataLoader(self.train_dataset, batch_size=config.train.batch_size,
                                       num_workers=config.data.num_workers,
                                       pin_memory=config.data.pin_memory and self.device.type == "cuda",
                                       collate_fn=self._build_lm_collate_fn(config))
        self.num_train_samples = self.train_dataset.total_samples
        self.train_sampler_epoch = 0
        self.train_loader_iter_idx = 0
        self.train_loader_iter = enumerate(self.train_loader)
        self._stream_offset = 0  # globally consumed samples before step 0 of this run

    def _next_train_batch(self):
        if getattr(self, "_stream_offset", None) is None:
            return super()._next_train_batch()
        try:
            idx, batch = next(self.train_loader_iter)
        except StopIteration:
            self.train_dataset.global_skip = 0
            self.train_dataset.set_epoch(self.train_dataset.epoch + 1)
            self.train_loader_iter = enumerate(self.train_loader)
            idx, batch = next(self.train_loader_iter)
        self.train_loader_iter_idx = idx + 1
        return batch

    def _stream_position(self, next_step: int) -> dict:
        consumed = self._stream_offset + next_step * self._global_samples_per_step()
        total = max(1, self.train_dataset.total_samples)
        return {"epoch": consumed // total, "global_skip": consumed % total}

    def save(self, step: int | None = None):
        if hasattr(self.train_dataset, "global_skip"):
            self._pending_dataset_state = self._stream_position((step or 0) + 1)
        super().save(step)

    def _checkpoint_extra_meta(self) -> dict:
        state = getattr(self, "_pending_dataset_state", None)
        return {"dataset_state": state} if state is not None else {}

    def _resume_from_checkpoint(self):
        super()._resume_from_checkpoint()
        meta = getattr(self, "_resumed_meta", None)
        if meta is None or not hasattr(self.train_dataset, "global_skip"):
            return
        state = meta.get("dataset_state")
        if state is None:
            return
        self.train_dataset.set_epoch(int(state["epoch"]))
        self.train_dataset.global_skip = int(state["global_skip"])
        self.train_loader_iter = enumerate(self.train_loader)
        consumed = int(state["epoch"]) * max(1, self.train_dataset.total_samples) + int(state["global_skip"])
        self._stream_offset = consumed - self.start_step * self._global_samples_per_step()
