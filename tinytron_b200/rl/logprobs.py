"""Token log-probabilities and masked reductions (reference: tinytron/rl/logprobs.py:8-123)."""
from __future__ import annotations

import torch
import torch.distributed as dist
import torch.nn.functional as F


def gather_log_probs(logits: torch.Tensor, token_ids: torch.Tensor) -> torch.Tensor:
    """log p(token_ids) for logits [..., V]."""
    if token_ids.shape == logits.shape:
        raise ValueError("token_ids should not include the vocab dimension")
    if token_ids.shape != logits.shape[:-1]:
        raise ValueError(f"token_ids shape {tuple(token_ids.shape)} must match logits shape {tuple(logits.shape[:-1])}")
    lp = F.log_softmax(logits.float(), dim=-1)
    return lp.gather(-1, token_ids.unsqueeze(-1)).squeeze(-1)


def causal_log_probs(logits: torch.Tensor, input_ids: torch.Tensor) -> torch.Tensor:
    if logits.dim() != 3 or input_ids.dim() != 2:
        raise ValueError("logits must be [B, T, V] and input_ids must be [B, T]")
    if logits.shape[:2] != input_ids.shape:
        raise ValueError("logits and input_ids must share batch and sequence dimensions")
    return gather_log_probs(logits[:, :-1], input_ids[:, 1:])


def response_log_probs(logits, sequences, response_mask):
    lp = causal_log_probs(logits, sequences)
    if response_mask.shape != lp.shape:
        raise ValueError(f"response_mask shape {tuple(response_mask.shape)} must match log_probs {tuple(lp.shape)}")
    return lp * response_mask.to(lp.dtype)


def masked_sum(values, mask, group=None):
    total = (values * mask.to(values.dtype)).sum()
    if group is not None:
        dist.all_reduce(total, op=dist.ReduceOp.SUM, group=group)
    return total


def masked_mean(values, mask, group=None, eps: float = 1e-8):
    m = mask.to(values.dtype)
    num, den = (values * m).sum(), m.sum()
    if group is not None:
        st = torch.stack([num, den])
        dist.all_reduce(st, op=dist.ReduceOp.SUM, group=group)
        num, den = st.unbind()
    return num / den.clamp_min(eps)


def sequence_log_probs(token_log_probs, mask, average: bool = False, group=None):
    m = mask.to(token_log_probs.dtype)
    logp = (token_log_probs * m).sum(-1)
    count = m.sum(-1)
    if group is not None:
        dist.all_reduce(logp, op=dist.ReduceOp.SUM, group=group)
        dist.all_reduce(count, op=dist.ReduceOp.SUM, group=group)
    return logp / count.clamp_min(1.0) if average else logp


def build_response_mask(sequences: torch.Tensor, prompt_len: int, eos_token_id: int | None = None) -> torch.Tensor:
    """Mask aligned to causal_log_probs(sequences) ([B, T-1]); response tokens up to and
    including the first EOS are 1."""
    if sequences.dim() != 2:
        raise ValueError("sequences must be [B, T]")
    if not 0 < prompt_len <= sequences.size(1):
        raise ValueError(f"prompt_len must be in [1, {sequences.size(1)}], got {prompt_len}")
    B, T = sequences.shape
    mask = torch.zeros(B, T - 1, dtype=torch.float32, device=sequences.device)
    mask[:, prompt_len - 1:] = 1.0
    if eos_token_id is None:
        return mask
    resp = sequences[:, prompt_len:]
    hits = resp.eq(eos_token_id)
    first = hits.float().argmax(-1)
    keep = torch.arange(resp.size(1), device=sequences.device)[None] <= first[:, None]
    keep = torch.where(hits.any(-1, keepdim=True), keep, torch.ones_like(keep))
    mask[:, prompt_len - 1:] = keep.to(mask.dtype)
    return mask
