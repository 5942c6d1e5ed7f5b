"""Per-token log-probabilities and masked reductions for RL objectives.

Public functions and their semantics follow the reference API
(tinytron/rl/logprobs.py:8-123): ``gather_log_probs``, ``causal_log_probs``,
``response_log_probs``, ``masked_sum``, ``masked_mean``, ``sequence_log_probs`` and
``build_response_mask``.  The implementation is organised around two B200 concerns:

* Memory.  A log-probability is ``logit[target] - logsumexp(logits)``.  The row
  log-sum-exp is formed in fp32 over row blocks (``_ROWS_PER_BLOCK`` rows at a time), so
  no fp32 copy of a ``[B, T, V]`` logits tensor (1.6 GB at 8K tokens x 50K vocab) is ever
  materialised; the backward rebuilds ``onehot - softmax`` block by block from the saved
  per-row log-sum-exp.  (The actor's own log-probs in the RL trainer skip logits
  entirely: ``GPT.token_log_probs`` runs the fused LM-head + cross-entropy kernel.)
* Collectives.  Every cross-rank reduction here packs all of its partial sums into ONE
  tensor and issues a single all-reduce (the reference issues one per quantity).
"""
from __future__ import annotations

import torch
import torch.distributed as dist

_ROWS_PER_BLOCK = 4096


def packed_all_reduce(parts: list[torch.Tensor], group=None) -> list[torch.Tensor]:
    """Sum-reduce several tensors over ``group`` with one collective.

    The tensors are flattened into one fp32 buffer (autograd flows through to each
    part unchanged, i.e. d(global sum)/d(local part) = 1), reduced once, and split back
    to the original shapes.  With ``group=None`` the parts are returned as they are."""
    if group is None:
        return parts
    shapes = [p.shape for p in parts]
    flat = torch.cat([p.reshape(-1).to(torch.float32) for p in parts])
    dist.all_reduce(flat, op=dist.ReduceOp.SUM, group=group)
    out, off = [], 0
    for p, s in zip(parts, shapes):
        n = p.numel()
        out.append(flat[off:off + n].view(s).to(p.dtype))
        off += n
    return out


class _TokenLogProb(torch.autograd.Function):
    """log softmax(logits)[target] over the last dim, computed in fp32 row blocks."""

    @staticmethod
    def forward(ctx, logits2d, targets1d):
        n = logits2d.shape[0]
        out = torch.empty(n, dtype=torch.float32, device=logits2d.device)
        lse = torch.empty(n, dtype=torch.float32, device=logits2d.device)
        for r0 in range(0, n, _ROWS_PER_BLOCK):
            blk = logits2d[r0:r0 + _ROWS_PER_BLOCK].float()
            lse[r0:r0 + blk.shape[0]] = torch.logsumexp(blk, dim=-1)
            picked = blk.gather(-1, targets1d[r0:r0 + blk.shape[0]].unsqueeze(-1)).squeeze(-1)
            out[r0:r0 + blk.shape[0]] = picked - lse[r0:r0 + blk.shape[0]]
        ctx.save_for_backward(logits2d, targets1d, lse)
        return out

    @staticmethod
    def backward(ctx, g):
        logits2d, targets1d, lse = ctx.saved_tensors
        grad = torch.empty_like(logits2d)
        for r0 in range(0, logits2d.shape[0], _ROWS_PER_BLOCK):
            r1 = min(r0 + _ROWS_PER_BLOCK, logits2d.shape[0])
            p = torch.exp(logits2d[r0:r1].float() - lse[r0:r1, None])  # softmax of the block
            p.neg_()
            p.scatter_add_(-1, targets1d[r0:r1, None], torch.ones(r1 - r0, 1, device=p.device))
            grad[r0:r1] = (p * g[r0:r1, None]).to(grad.dtype)  # g * (onehot - softmax)
        return grad, None


def gather_log_probs(logits: torch.Tensor, token_ids: torch.Tensor) -> torch.Tensor:
    """log p(token_ids) under softmax(logits) for logits ``[..., V]`` and ids ``[...]``
    (fp32 result, differentiable with respect to ``logits``)."""
    if token_ids.dim() == logits.dim():
        raise ValueError("token_ids must not carry a vocabulary dimension: expected shape "
                         f"{tuple(logits.shape[:-1])}, got {tuple(token_ids.shape)}")
    if tuple(token_ids.shape) != tuple(logits.shape[:-1]):
        raise ValueError(f"token_ids shape {tuple(token_ids.shape)} does not match the leading dims "
                         f"{tuple(logits.shape[:-1])} of logits")
    lead = token_ids.shape
    flat = _TokenLogProb.apply(logits.reshape(-1, logits.shape[-1]), token_ids.reshape(-1).long())
    return flat.view(lead)


def causal_log_probs(logits: torch.Tensor, input_ids: torch.Tensor) -> torch.Tensor:
    """Log-probs of ``input_ids[:, 1:]`` from next-token logits ``[B, T, V]`` (result ``[B, T-1]``)."""
    if logits.dim() != 3 or input_ids.dim() != 2:
        raise ValueError(f"expected logits [B, T, V] and input_ids [B, T], got {tuple(logits.shape)} and "
                         f"{tuple(input_ids.shape)}")
    if tuple(logits.shape[:2]) != tuple(input_ids.shape):
        raise ValueError(f"logits {tuple(logits.shape)} and input_ids {tuple(input_ids.shape)} disagree on "
                         "batch or sequence length")
    return gather_log_probs(logits[:, :-1], input_ids[:, 1:])


def response_log_probs(logits: torch.Tensor, sequences: torch.Tensor, response_mask: torch.Tensor) -> torch.Tensor:
    """``causal_log_probs`` with non-response positions zeroed (mask aligned to ``sequences[:, 1:]``)."""
    lp = causal_log_probs(logits, sequences)
    if tuple(response_mask.shape) != tuple(lp.shape):
        raise ValueError(f"response_mask {tuple(response_mask.shape)} must align with the log-probs "
                         f"{tuple(lp.shape)} (i.e. with sequences[:, 1:])")
    return lp * response_mask.to(lp.dtype)


def masked_sum(values: torch.Tensor, mask: torch.Tensor, group=None) -> torch.Tensor:
    """Sum of ``values * mask`` (over ``group`` too, when given)."""
    (total,) = packed_all_reduce([(values * mask.to(values.dtype)).sum()], group)
    return total


def masked_mean(values: torch.Tensor, mask: torch.Tensor, group=None, eps: float = 1e-8) -> torch.Tensor:
    """sum(values * mask) / sum(mask), both sums taken over ``group`` in one collective."""
    m = mask.to(values.dtype)
    num, den = packed_all_reduce([(values * m).sum(), m.sum()], group)
    return num / den.clamp_min(eps)


def sequence_log_probs(token_log_probs: torch.Tensor, mask: torch.Tensor, average: bool = False,
                       group=None) -> torch.Tensor:
    """Per-sequence log-prob: masked sum over the last dim (or the masked mean with
    ``average``).  With a ``group`` (sequence-parallel shards) the per-rank partial sums
    and counts are reduced together."""
    m = mask.to(token_log_probs.dtype)
    total, count = packed_all_reduce([(token_log_probs * m).sum(-1), m.sum(-1)], group)
    return total / count.clamp_min(1.0) if average else total


def build_response_mask(sequences: torch.Tensor, prompt_len: int, eos_token_id: int | None = None) -> torch.Tensor:
    """fp32 mask ``[B, T-1]`` aligned to ``causal_log_probs(sequences)``: 1 on generated
    tokens, 0 on the prompt; with ``eos_token_id``, generated tokens after a sequence's
    first EOS are 0 (the EOS itself stays 1)."""
    if sequences.dim() != 2:
        raise ValueError(f"sequences must be [B, T], got {tuple(sequences.shape)}")
    T = sequences.size(1)
    if not 1 <= prompt_len <= T:
        raise ValueError(f"prompt_len {prompt_len} is outside [1, {T}]")
    pos = torch.arange(T - 1, device=sequences.device)
    mask = (pos >= prompt_len - 1).expand(sequences.size(0), -1)
    if eos_token_id is not None:
        # an EOS strictly before a generated position (inclusive count minus the token itself)
        is_eos = sequences[:, 1:].eq(eos_token_id) & mask
        seen_before = (is_eos.cumsum(-1) - is_eos.long()) > 0
        mask = mask & ~seen_before
    return mask.to(torch.float32)
