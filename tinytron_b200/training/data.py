"""Mock dataset, LM collate and batch helpers (reference: tinytron/training/trainer.py:93-192)."""
from __future__ import annotations

import torch
from torch.nn.utils.rnn import pad_sequence
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


def build_lm_collate_fn(seq_len: int, sp_world_size: int, pad_token_id: int = 0, ignore_index: int = IGNORE_INDEX):
    """Collate to [B, T]; T is padded up to a multiple of the SP size (labels padded
    with ignore_index); items without labels are shifted by one."""

    def _1d(v) -> torch.Tensor:
        t = v if torch.is_tensor(v) else torch.tensor(v, dtype=torch.long)
        return t.to(torch.long).view(-1)

    def collate(batch):
        xs, ys = [], []
        for item in batch:
            if "labels" in item:
                x, y = _1d(item["input_ids"]), _1d(item["labels"])
            else:
                tok = _1d(item["input_ids"])
                x, y = tok[:-1], tok[1:]
            n = min(x.numel(), y.numel(), seq_len)
            xs.append(x[:n])
            ys.append(y[:n])
        max_len = max((x.numel() for x in xs), default=0)
        if max_len == 0:
            raise ValueError("Encountered an empty language-modeling batch.")
        target = min(max_len, seq_len)
        if target % sp_world_size:
            target += sp_world_size - target % sp_world_size
        if target > seq_len:
            raise ValueError(f"Batch max sequence length {max_len} cannot be padded to sep_size={sp_world_size} "
                             f"within seq_len={seq_len}.")
        x = pad_sequence([t[:target] for t in xs], batch_first=True, padding_value=pad_token_id)
        y = pad_sequence([t[:target] for t in ys], batch_first=True, padding_value=ignore_index)
        if x.size(1) < target:
            x = torch.nn.functional.pad(x, (0, target - x.size(1)), value=pad_token_id)
            y = torch.nn.functional.pad(y, (0, target - y.size(1)), value=ignore_index)
        return {"input_ids": x, "labels": y, "valid_token_count": (y != ignore_index).sum(),
                "padded_token_count": torch.tensor(x.numel(), dtype=torch.long)}

    return collate
