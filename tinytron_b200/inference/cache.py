"""Paged KV cache with a real page table (reference API: tinytron/inference/cache.py:11-97).

Each layer owns a pool of fixed-size pages ``[num_pages, page_size, H_kv_local, D]``
(token-major inside a page, unexpanded kv heads) and a page table
``[batch, pages_per_seq]`` (int32, -1 = unmapped).  Pages are taken from a free list
as sequences grow, so sequences of different lengths share one pool.  The reference
API is kept: ``append(k, v)`` with [B, H, T, D] tensors returns the previous length,
``get_kv()`` returns contiguous [B, H, L, D] views for generic attention, and
``current_length`` is the common length.  Decode kernels read pages directly via
``page_table``.  ``PagedKVCache.contiguous(...)`` builds the same object with
one page per sequence (a contiguous cache).
"""
from __future__ import annotations

import math

import torch

from tinytron_b200.parallel import parallel_state


class LayerPagedKVCache:
    def __init__(self, batch_size: int, num_heads: int, head_dim: int, max_seq_len: int, page_size: int,
                 device, dtype, num_pages: int | None = None):
        if page_size <= 0:
            raise ValueError(f"page_size must be positive, got {page_size}")
        self.batch_size = batch_size
        self.num_heads = num_heads
        self.head_dim = head_dim
        self.max_seq_len = max_seq_len
        self.page_size = page_size
        self.pages_per_seq = math.ceil(max_seq_len / page_size)
        total = num_pages if num_pages is not None else batch_size * self.pages_per_seq
        self.k_pages = torch.empty(total, page_size, num_heads, head_dim, device=device, dtype=dtype)
        self.v_pages = torch.empty_like(self.k_pages)
        self.page_table = torch.full((batch_size, self.pages_per_seq), -1, dtype=torch.int32, device=device)
        self._host_table = [[-1] * self.pages_per_seq for _ in range(batch_size)]
        self._free = list(range(total - 1, -1, -1))
        self.current_length = 0
        self.seq_lens = [0] * batch_size
        # Device copy of the common length: the fused decode kernels read positions
        # from it, so a decode step captured in a CUDA graph stays valid on replay.
        self.len_dev = torch.zeros(1, dtype=torch.int32, device=device)
        self._scratch = None  # (splits, o_part, ml_part) for decode attention

    def _ensure_pages(self, new_len: int) -> None:
        need = math.ceil(new_len / self.page_size)
        changed = False
        for b in range(self.batch_size):
            row = self._host_table[b]
            for p in range(need):
                if row[p] < 0:
                    if not self._free:
                        raise RuntimeError("KV cache page pool exhausted")
                    row[p] = self._free.pop()
                    changed = True
        if changed:
            self.page_table.copy_(torch.tensor(self._host_table, dtype=torch.int32))

    def reserve(self, length: int) -> None:
        """Map pages for positions [0, length) of every sequence now (no page is
        allocated during later appends; required before capturing a decode graph)."""
        if length > self.max_seq_len:
            raise ValueError(f"KV cache overflow: requested sequence length {length}, max supported is "
                             f"{self.max_seq_len}")
        self._ensure_pages(length)

    # ---------------------------------------------------------------- fused CUDA path
    def append_rope(self, qkv: torch.Tensor, B: int, T: int, Hq: int, Hkv: int, D: int, theta: float) -> torch.Tensor:
        """qkv [B*T, (Hq+2Hkv)*D] bf16 -> rotated q [B*T, Hq*D]; K (rotated) and V are
        written into the pages at positions len + t (len read on the device).  Call
        :meth:`advance` after the attention that reads them."""
        from tinytron_b200.ops import _ext
        from tinytron_b200.ops.rope import rope_tables

        end = self.current_length + T
        if end > self.max_seq_len:
            raise ValueError(f"KV cache overflow: requested sequence length {end}, max supported is {self.max_seq_len}")
        self._ensure_pages(end)
        cos, sin = rope_tables(D, theta, self.max_seq_len, qkv.device)
        q = torch.empty(B * T, Hq * D, dtype=torch.bfloat16, device=qkv.device)
        _ext.load().decode_rope_append(qkv, B, T, Hq, Hkv, D, self.len_dev, 0, cos, sin, q, self.k_pages,
                                       self.v_pages, self.page_table)
        return q

    def attend_decode(self, q: torch.Tensor, scale: float) -> torch.Tensor:
        """One new token per sequence: q [B, Hq, D] (rotated, already appended) ->
        attention over keys [0, len + 1) -> [B, Hq*D] bf16."""
        from tinytron_b200.ops import _ext

        C = _ext.load()
        B, Hq, D = q.shape
        if self._scratch is None or self._scratch[1].numel() < B * Hq * self._scratch[0] * D:
            splits = int(C.decode_num_splits(self.max_seq_len))
            self._scratch = (splits, torch.empty(B * Hq * splits * D, device=q.device),
                             torch.empty(B * Hq * splits * 2, device=q.device))
        splits, o_part, ml_part = self._scratch
        out = torch.empty(B, Hq * D, dtype=torch.bfloat16, device=q.device)
        C.decode_attention(q, self.k_pages, self.v_pages, self.page_table, self.len_dev, 1, splits, scale, o_part,
                           ml_part, out)
        return out

    def advance(self, T: int) -> int:
        """Commit T appended positions (host length and the device copy)."""
        prev = self.current_length
        self.current_length += T
        self.seq_lens = [self.current_length] * self.batch_size
        self.len_dev.add_(T)
        return prev

    def set_length(self, length: int) -> None:
        """Host and device length := length (e.g. after CUDA-graph replays advanced the
        device copy only)."""
        self.current_length = length
        self.seq_lens = [length] * self.batch_size
        self.len_dev.fill_(length)

    def append(self, k: torch.Tensor, v: torch.Tensor) -> int:
        T = k.size(2)
        end = self.current_length + T
        if end > self.max_seq_len:
            raise ValueError(f"KV cache overflow: requested sequence length {end}, max supported is {self.max_seq_len}")
        self._ensure_pages(end)
        pos = torch.arange(self.current_length, end, device=self.k_pages.device)
        page = self.page_table[:, (pos // self.page_size)].long()  # [B, T]
        off = (pos % self.page_size).expand_as(page)
        self.k_pages[page, off] = k.transpose(1, 2).to(self.k_pages.dtype)
        self.v_pages[page, off] = v.transpose(1, 2).to(self.v_pages.dtype)
        prev = self.current_length
        self.current_length = end
        self.seq_lens = [end] * self.batch_size
        self.len_dev.fill_(end)
        return prev

    def gather_tokens(self, length: int | None = None):
        """[B, L, H, D] K and V in token order."""
        L = self.current_length if length is None else length
        n = math.ceil(L / self.page_size)
        pt = self.page_table[:, :n].long()
        k = self.k_pages[pt].reshape(self.batch_size, n * self.page_size, self.num_heads, self.head_dim)[:, :L]
        v = self.v_pages[pt].reshape(self.batch_size, n * self.page_size, self.num_heads, self.head_dim)[:, :L]
        return k, v

    def get_kv(self):
        k, v = self.gather_tokens()
        return k.transpose(1, 2), v.transpose(1, 2)

    def reset(self) -> None:
        self.page_table.fill_(-1)
        self._host_table = [[-1] * self.pages_per_seq for _ in range(self.batch_size)]
        self._free = list(range(self.k_pages.size(0) - 1, -1, -1))
        self.current_length = 0
        self.seq_lens = [0] * self.batch_size
        self.len_dev.zero_()


class PagedKVCache:
    def __init__(self, layer_caches: list[LayerPagedKVCache]) -> None:
        self._layer_caches = layer_caches

    @staticmethod
    def local_kv_heads(model_config) -> int:
        """kv heads stored per rank: all kv heads, or the SEP rank's share in head-parallel decode."""
        sep = parallel_state.get_sep_world_size()
        Hq, Hkv = model_config.num_attention_heads, model_config.num_key_value_heads
        if sep <= 1:
            return Hkv
        if Hq % sep:
            raise ValueError(f"num_attention_heads ({Hq}) must be divisible by sep_size ({sep})")
        hq_l, G = Hq // sep, Hq // Hkv
        if Hkv % sep == 0:
            return Hkv // sep
        if G % hq_l == 0:
            return 1
        return hq_l  # non-uniform q->kv mapping: kv heads expanded to the local q heads

    @classmethod
    def from_model_config(cls, model_config, batch_size: int, page_size: int, device, dtype,
                          max_seq_len: int | None = None) -> "PagedKVCache":
        heads = cls.local_kv_heads(model_config)
        hd = model_config.hidden_size // model_config.num_attention_heads
        L = max_seq_len or model_config.block_size
        return cls([LayerPagedKVCache(batch_size, heads, hd, L, page_size, device, dtype)
                    for _ in range(model_config.num_layer)])

    @classmethod
    def contiguous(cls, model_config, batch_size: int, device, dtype, max_seq_len: int | None = None):
        L = max_seq_len or model_config.block_size
        return cls.from_model_config(model_config, batch_size, L, device, dtype, max_seq_len=L)

    def reserve(self, length: int) -> None:
        for c in self._layer_caches:
            c.reserve(length)

    def set_length(self, length: int) -> None:
        for c in self._layer_caches:
            c.set_length(length)

    @property
    def current_length(self) -> int:
        return self._layer_caches[0].current_length if self._layer_caches else 0

    def get_layer_cache(self, layer_idx: int) -> LayerPagedKVCache:
        return self._layer_caches[layer_idx]

    def __len__(self):
        return len(self._layer_caches)
