"""Policy objectives for RL fine-tuning: the k3 KL estimator, vanilla policy gradient,
the PPO clipped surrogate, GRPO (PPO on group-normalised advantages plus an optional
KL penalty) and DPO.  Names, arguments, metric keys and values follow the reference
(tinytron/rl/losses.py:11-125).

Every masked statistic an objective reports is reduced in one pass: the per-token
quantities are summed under the mask locally and, with a sequence-parallel ``group``,
all of them (and the mask count) cross ranks in a single packed all-reduce.  PPO, for
instance, needs one collective for its loss, clip fraction and mean ratio together.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from .logprobs import packed_all_reduce
from .types import RLLossOutput


def _per_token(advantages: torch.Tensor, log_probs: torch.Tensor) -> torch.Tensor:
    """Advantages shaped like ``log_probs`` (per token) or like its batch dims (per
    sequence, broadcast over the last dim)."""
    if advantages.shape == log_probs.shape:
        return advantages
    if advantages.shape == log_probs.shape[:-1]:
        return advantages[..., None]
    raise ValueError(f"advantages {tuple(advantages.shape)} fit neither the per-token shape "
                     f"{tuple(log_probs.shape)} nor the per-sequence shape {tuple(log_probs.shape[:-1])}")


def _masked_means(values: list[torch.Tensor], mask: torch.Tensor, group=None, eps: float = 1e-8):
    """[sum(v * mask) / sum(mask) for v in values], all sums reduced in one collective.
    Gradients flow to every entry of ``values`` that requires them."""
    m = mask.to(values[0].dtype)
    sums = torch.stack([(v * m).sum() for v in values] + [m.sum()])
    (sums,) = packed_all_reduce([sums], group)
    den = sums[-1].clamp_min(eps)
    return [sums[i] / den for i in range(len(values))]


def approx_kl(policy_log_probs: torch.Tensor, reference_log_probs: torch.Tensor, mask: torch.Tensor,
              group=None) -> torch.Tensor:
    """Masked mean of the k3 estimator exp(d) - d - 1, d = log p_ref - log p_policy (>= 0)."""
    d = reference_log_probs - policy_log_probs
    (kl,) = _masked_means([torch.expm1(d) - d], mask, group)
    return kl


def policy_gradient_loss(log_probs: torch.Tensor, advantages: torch.Tensor, mask: torch.Tensor,
                         group=None) -> RLLossOutput:
    """REINFORCE-style loss: -masked_mean(log_probs * advantages)."""
    (obj,) = _masked_means([log_probs * _per_token(advantages, log_probs)], mask, group)
    loss = -obj
    return RLLossOutput(loss=loss, metrics={"pg_loss": loss.detach()})


def _ppo_terms(log_probs, old_log_probs, advantages, clip_range):
    adv = _per_token(advantages, log_probs)
    ratio = torch.exp(log_probs - old_log_probs)
    surrogate = ratio * adv
    clipped = ratio.clamp(1.0 - clip_range, 1.0 + clip_range) * adv
    objective = torch.minimum(surrogate, clipped)
    was_clipped = (surrogate != objective).to(log_probs.dtype)
    return objective, was_clipped, ratio


def ppo_policy_loss(log_probs: torch.Tensor, old_log_probs: torch.Tensor, advantages: torch.Tensor,
                    mask: torch.Tensor, clip_range: float = 0.2, group=None) -> RLLossOutput:
    """PPO clipped surrogate; metrics: the loss, the clipped-token fraction and the mean ratio."""
    objective, was_clipped, ratio = _ppo_terms(log_probs, old_log_probs, advantages, clip_range)
    obj, frac, mean_ratio = _masked_means([objective, was_clipped.detach(), ratio.detach()], mask, group)
    loss = -obj
    return RLLossOutput(loss=loss, metrics={"ppo_loss": loss.detach(), "clip_frac": frac.detach(),
                                            "mean_ratio": mean_ratio.detach()})


def grpo_loss(log_probs: torch.Tensor, old_log_probs: torch.Tensor, advantages: torch.Tensor, mask: torch.Tensor,
              reference_log_probs: torch.Tensor | None = None, clip_range: float = 0.2, kl_coef: float = 0.0,
              group=None) -> RLLossOutput:
    """PPO surrogate plus ``kl_coef`` x the k3 KL to a reference policy (when given and
    ``kl_coef > 0``); the KL rides in the same collective as the PPO statistics."""
    objective, was_clipped, ratio = _ppo_terms(log_probs, old_log_probs, advantages, clip_range)
    with_kl = reference_log_probs is not None and kl_coef > 0.0
    terms = [objective, was_clipped.detach(), ratio.detach()]
    if with_kl:
        d = reference_log_probs - log_probs
        terms.append(torch.expm1(d) - d)
    means = _masked_means(terms, mask, group)
    loss = -means[0]
    metrics = {"ppo_loss": loss.detach(), "clip_frac": means[1].detach(), "mean_ratio": means[2].detach()}
    if with_kl:
        loss = loss + kl_coef * means[3]
        metrics["kl"] = means[3].detach()
    return RLLossOutput(loss=loss, metrics=metrics)


def dpo_loss(chosen_log_probs: torch.Tensor, rejected_log_probs: torch.Tensor,
             reference_chosen_log_probs: torch.Tensor, reference_rejected_log_probs: torch.Tensor,
             beta: float = 0.1) -> RLLossOutput:
    """Direct preference optimisation: -log sigmoid(beta * (policy margin - reference margin))."""
    chosen_reward = beta * (chosen_log_probs - reference_chosen_log_probs)
    rejected_reward = beta * (rejected_log_probs - reference_rejected_log_probs)
    margin = chosen_reward - rejected_reward  # = beta * (policy margin - reference margin)
    loss = F.softplus(-margin).mean()  # -log sigmoid(x) = softplus(-x)
    m = margin.detach()
    return RLLossOutput(loss=loss, metrics={
        "dpo_loss": loss.detach(),
        "reward_accuracy": (m > 0).float().mean(),
        "reward_margin": m.mean(),
        "chosen_reward": chosen_reward.detach().mean(),
        "rejected_reward": rejected_reward.detach().mean(),
    })
