"""Rollout batches and group-relative advantages (API and semantics of the reference's
tinytron/rl/rollout.py:9-64).

A rollout batch is derived from the generated ``sequences`` (prompt + completion) in
one pass: the response mask (EOS-aware), the labels (the next tokens with every
non-action position set to ``ignore_index``) and, when given, the sampler's per-token
log-probs left-padded with zeros so every per-token tensor is aligned to
``sequences[:, 1:]``.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from .logprobs import build_response_mask
from .types import RolloutBatch


def make_rollout_batch(prompts: torch.Tensor, sequences: torch.Tensor, old_log_probs: torch.Tensor | None = None,
                       eos_token_id: int | None = None, ignore_index: int = -100) -> RolloutBatch:
    """Assemble a :class:`RolloutBatch` from prompts ``[B, P]`` and sequences ``[B, P + N]``;
    ``old_log_probs`` ``[B, N]`` are the sampler's log-probs of the N generated tokens."""
    if prompts.dim() != 2 or sequences.dim() != 2:
        raise ValueError(f"prompts and sequences must be 2-D [B, T], got {tuple(prompts.shape)} and "
                         f"{tuple(sequences.shape)}")
    B, P = prompts.shape
    if sequences.size(0) != B:
        raise ValueError(f"batch sizes differ: {B} prompts vs {sequences.size(0)} sequences")
    if sequences.size(1) < P:
        raise ValueError(f"sequences (length {sequences.size(1)}) must start with the {P}-token prompt")
    mask = build_response_mask(sequences, prompt_len=P, eos_token_id=eos_token_id)
    labels = torch.where(mask.bool(), sequences[:, 1:], torch.full_like(sequences[:, 1:], ignore_index))
    n_gen = sequences.size(1) - P
    aligned_old = None
    if old_log_probs is not None:
        if tuple(old_log_probs.shape) != (B, n_gen):
            raise ValueError(f"old_log_probs {tuple(old_log_probs.shape)} must cover the generated tokens "
                             f"({B}, {n_gen})")
        aligned_old = F.pad(old_log_probs.to(mask.dtype), (P - 1, 0))  # zeros under the prompt
    return RolloutBatch(
        prompts=prompts,
        responses=sequences[:, P:],
        sequences=sequences,
        labels=labels,
        response_mask=mask,
        prompt_lens=torch.full((B,), P, dtype=torch.long, device=sequences.device),
        response_lens=mask[:, P - 1:].sum(-1).long(),
        old_log_probs=aligned_old,
    )


def group_advantages(rewards: torch.Tensor, group_size: int, eps: float = 1e-6) -> torch.Tensor:
    """GRPO advantages: each reward minus its group's mean, over the group's population
    standard deviation (floored at ``eps``); groups are consecutive runs of ``group_size``."""
    if rewards.dim() != 1:
        raise ValueError(f"rewards must be 1-D [B], got {tuple(rewards.shape)}")
    if group_size < 1 or rewards.numel() % group_size:
        raise ValueError(f"{rewards.numel()} rewards cannot be split into groups of {group_size}")
    grouped = rewards.view(-1, group_size)
    var, mean = torch.var_mean(grouped, dim=-1, correction=0, keepdim=True)
    return ((grouped - mean) / var.sqrt().clamp_min(eps)).view_as(rewards)
