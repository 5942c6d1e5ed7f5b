"""Rollout batches and group advantages (reference: tinytron/rl/rollout.py:9-64)."""
from __future__ import annotations

import torch

from .logprobs import build_response_mask
from .types import RolloutBatch


def make_rollout_batch(prompts, sequences, old_log_probs=None, eos_token_id=None, ignore_index: int = -100):
    if prompts.dim() != 2 or sequences.dim() != 2:
        raise ValueError("prompts and sequences must be [B, T]")
    if prompts.size(0) != sequences.size(0):
        raise ValueError("prompts and sequences must share batch size")
    P = prompts.size(1)
    if sequences.size(1) < P:
        raise ValueError("sequences must include the prompt prefix")
    mask = build_response_mask(sequences, prompt_len=P, eos_token_id=eos_token_id)
    labels = sequences[:, 1:].clone().masked_fill(mask == 0, ignore_index)
    old_full = None
    if old_log_probs is not None:
        tok_mask = mask[:, P - 1:]
        if old_log_probs.shape != tok_mask.shape:
            raise ValueError("old_log_probs must be aligned to response tokens")
        old_full = torch.zeros_like(mask)
        old_full[:, P - 1:] = old_log_probs.to(old_full.dtype)
    return RolloutBatch(prompts=prompts, responses=sequences[:, P:], sequences=sequences, labels=labels,
                        response_mask=mask,
                        prompt_lens=torch.full((sequences.size(0),), P, dtype=torch.long, device=sequences.device),
                        response_lens=mask[:, P - 1:].sum(-1).long(), old_log_probs=old_full)


def group_advantages(rewards: torch.Tensor, group_size: int, eps: float = 1e-6) -> torch.Tensor:
    """(r - mean_group) / std_group (population std, clamped)."""
    if rewards.dim() != 1:
        raise ValueError("rewards must be [B]")
    if group_size <= 0 or rewards.numel() % group_size:
        raise ValueError("rewards length must be divisible by group_size")
    g = rewards.view(-1, group_size)
    return ((g - g.mean(-1, keepdim=True)) / g.std(-1, unbiased=False, keepdim=True).clamp_min(eps)).reshape_as(rewards)
