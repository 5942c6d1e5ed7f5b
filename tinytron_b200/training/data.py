"""Mock dataset and the LM collate function (capabilities of the reference's
tinytron/training/trainer.py:93-192).  ``MockDataset`` reproduces the reference's token
stream exactly (same seeding rule per sample), so loss curves compare directly."""
from __future__ import annotations

import torch
from torch.utils.data import Dataset

IGNORE_INDEX = -100


class MockDataset(Dataset):
    """Uniform random token sequences.  With ``deterministic`` each sample depends only
    on its global index (identical tokens across parallel layouts); otherwise the
    global RNG is used, as in the reference (trainer.py:96-117)."""

    def __init__(self, length: int, seq_len: int, vocab_size: int = 50304, deterministic: bool = False,
                 base_seed: int = 0, seed_offset: int = 0):
        self.length = length
        self.seq_len = seq_len
        self.vocab_size = vocab_size
        self.deterministic = deterministic
        self.base_seed = int(base_seed)
        self.seed_offset = int(seed_offset)

    def __len__(self):
        return self.length

    def __getitem__(self, idx):
        if self.deterministic:
            g = torch.Generator(device="cpu")
            g.manual_seed(self.base_seed + self.seed_offset + int(idx))
            data = torch.randint(0, self.vocab_size, (self.seq_len + 1,), dtype=torch.long, generator=g)
        else:
            data = torch.randint(0, self.vocab_size, (self.seq_len + 1,), dtype=torch.long)
        return {"input_ids": data[:self.seq_len], "labels": data[1:self.seq_len + 1]}


class LMCollator:
    """Batches variable-length LM samples into ``[B, T]`` ``input_ids`` / ``labels``.

    Each sample is ``{"input_ids", "labels"}`` (already shifted) or ``{"input_ids"}``
    alone (shifted here: inputs drop the last token, labels the first), and is cut to
    ``seq_len``.  T is the longest sample rounded up to a multiple of the SEP size, so the
    batch splits into equal sequence chunks; it may not exceed ``seq_len``.  The output
    rows are written into two preallocated tensors (inputs padded with ``pad_token_id``,
    labels with ``ignore_index``) with no per-sample padding pass.  A class rather than
    a closure so that DataLoader worker processes can pickle it.  Output keys and
    padding rules follow the reference collate (tinytron/training/trainer.py:145-192)."""

    def __init__(self, seq_len: int, sp_world_size: int, pad_token_id: int = 0, ignore_index: int = IGNORE_INDEX):
        self.seq_len = int(seq_len)
        self.sp = max(1, int(sp_world_size))
        self.pad_token_id = int(pad_token_id)
        self.ignore_index = int(ignore_index)

    @staticmethod
    def _tokens(v) -> torch.Tensor:
        return (v if torch.is_tensor(v) else torch.as_tensor(v)).reshape(-1).long()

    def _pair(self, item) -> tuple[torch.Tensor, torch.Tensor]:
        ids = self._tokens(item["input_ids"])
        if "labels" in item:
            x, y = ids, self._tokens(item["labels"])
        else:
            x, y = ids[:-1], ids[1:]
        n = min(x.numel(), y.numel(), self.seq_len)
        return x[:n], y[:n]

    def __call__(self, batch):
        pairs = [self._pair(item) for item in batch]
        longest = max((x.numel() for x, _ in pairs), default=0)
        if longest == 0:
            raise ValueError("cannot collate a batch whose samples are all empty")
        width = -(-longest // self.sp) * self.sp  # round up to a multiple of the SEP size
        if width > self.seq_len:
            raise ValueError(f"the longest sample ({longest} tokens) rounds up to {width} for sep_size={self.sp}, "
                             f"more than seq_len={self.seq_len}")
        x = torch.full((len(pairs), width), self.pad_token_id, dtype=torch.long)
        y = torch.full((len(pairs), width), self.ignore_index, dtype=torch.long)
        for row, (a, b) in enumerate(pairs):
            x[row, :a.numel()] = a
            y[row, :b.numel()] = b
        return {"input_ids": x, "labels": y, "valid_token_count": (y != self.ignore_index).sum(),
                "padded_token_count": torch.tensor(x.numel(), dtype=torch.long)}


def build_lm_collate_fn(seq_len: int, sp_world_size: int, pad_token_id: int = 0, ignore_index: int = IGNORE_INDEX):
    """The trainer's collate function (an :class:`LMCollator`)."""
    return LMCollator(seq_len, sp_world_size, pad_token_id, ignore_index)
