"""RoPE cos/sin tables and the reference-semantics RoPE for the CPU path.

HF Llama/Qwen-style half-split rotation as in the reference
(tinytron/model/modules/attn.py:13-63).  The reference rebuilds cos/sin on every
forward; here they are computed once per (head_dim, theta, device) in fp32 with the
same arithmetic (fp32 inv_freq, fp32 position*inv_freq product) and cached.  Only
the first half of the reference's ``cat(freqs, freqs)`` is stored ([max_pos, d/2]).
"""
from __future__ import annotations

import torch

_TABLES: dict = {}


def rope_tables(head_dim: int, theta: float, max_len: int, device) -> tuple[torch.Tensor, torch.Tensor]:
    device = torch.device(device)
    key = (head_dim, float(theta), device)
    cached = _TABLES.get(key)
    if cached is not None and cached[0].size(0) >= max_len:
        return cached
    n = max(max_len, 4096 if cached is None else 2 * cached[0].size(0))
    inv_freq = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float32, device=device) / head_dim))
    pos = torch.arange(n, device=device, dtype=torch.float32)
    freqs = pos[:, None] * inv_freq[None, :]
    tables = (freqs.cos().contiguous(), freqs.sin().contiguous())
    _TABLES[key] = tables
    return tables


def rope_reference(q: torch.Tensor, k: torch.Tensor, position_ids: torch.Tensor, theta: float = 10000.0):
    """Reference-semantics RoPE on [B, H, T, D] tensors (fp32-friendly CPU path)."""
    B, H, T, D = q.shape
    assert D % 2 == 0, f"head_dim must be even for RoPE, got {D}"
    inv_freq = 1.0 / (theta ** (torch.arange(0, D, 2, dtype=torch.float32, device=q.device) / D))
    if position_ids.dim() == 1:
        position_ids = position_ids.unsqueeze(0).expand(B, -1)
    elif position_ids.size(0) == 1 and B > 1:
        position_ids = position_ids.expand(B, -1)
    freqs = position_ids.float()[..., None] * inv_freq
    emb = torch.cat((freqs, freqs), dim=-1)
    cos = emb.cos().unsqueeze(1).to(q.dtype)
    sin = emb.sin().unsqueeze(1).to(q.dtype)

    def rot(x):
        return torch.cat((-x[..., D // 2:], x[..., : D // 2]), dim=-1)

    return q * cos + rot(q) * sin, k * cos + rot(k) * sin
