"""Policy losses (reference: tinytron/rl/losses.py:11-125): k3 KL estimate, vanilla PG,
PPO clipped objective, GRPO (= PPO with group-normalised advantages + optional KL),
and DPO."""
from __future__ import annotations

import torch
import torch.nn.functional as F

from .logprobs import masked_mean
from .types import RLLossOutput


def _align(adv, lp):
    if adv.shape == lp.shape:
        return adv
    if adv.shape == lp.shape[:-1]:
        return adv.unsqueeze(-1)
    raise ValueError(f"advantages shape {tuple(adv.shape)} must match log_probs {tuple(lp.shape)} or batch shape")


def approx_kl(policy_log_probs, reference_log_probs, mask, group=None):
    r = reference_log_probs - policy_log_probs
    return masked_mean(torch.exp(r) - r - 1.0, mask, group=group)


def policy_gradient_loss(log_probs, advantages, mask, group=None) -> RLLossOutput:
    loss = -masked_mean(log_probs * _align(advantages, log_probs), mask, group=group)
    return RLLossOutput(loss=loss, metrics={"pg_loss": loss.detach()})


def ppo_policy_loss(log_probs, old_log_probs, advantages, mask, clip_range: float = 0.2, group=None) -> RLLossOutput:
    adv = _align(advantages, log_probs)
    ratio = torch.exp(log_probs - old_log_probs)
    unclipped = ratio * adv
    clipped = torch.clamp(ratio, 1.0 - clip_range, 1.0 + clip_range) * adv
    obj = torch.minimum(unclipped, clipped)
    loss = -masked_mean(obj, mask, group=group)
    with torch.no_grad():
        clip_frac = masked_mean((unclipped != obj).to(log_probs.dtype), mask, group=group)
        mean_ratio = masked_mean(ratio, mask, group=group)
    return RLLossOutput(loss=loss, metrics={"ppo_loss": loss.detach(), "clip_frac": clip_frac, "mean_ratio": mean_ratio})


def grpo_loss(log_probs, old_log_probs, advantages, mask, reference_log_probs=None, clip_range: float = 0.2,
              kl_coef: float = 0.0, group=None) -> RLLossOutput:
    out = ppo_policy_loss(log_probs, old_log_probs, advantages, mask, clip_range=clip_range, group=group)
    loss, metrics = out.loss, dict(out.metrics)
    if reference_log_probs is not None and kl_coef > 0.0:
        kl = approx_kl(log_probs, reference_log_probs, mask, group=group)
        loss = loss + kl_coef * kl
        metrics["kl"] = kl.detach()
    return RLLossOutput(loss=loss, metrics=metrics)


def dpo_loss(chosen_log_probs, rejected_log_probs, reference_chosen_log_probs, reference_rejected_log_probs,
             beta: float = 0.1) -> RLLossOutput:
    margin = (chosen_log_probs - rejected_log_probs) - (reference_chosen_log_probs - reference_rejected_log_probs)
    loss = -F.logsigmoid(beta * margin).mean()
    with torch.no_grad():
        cr = beta * (chosen_log_probs - reference_chosen_log_probs)
        rr = beta * (rejected_log_probs - reference_rejected_log_probs)
        m = cr - rr
    return RLLossOutput(loss=loss, metrics={"dpo_loss": loss.detach(), "reward_accuracy": m.gt(0).float().mean(),
                                            "reward_margin": m.mean(), "chosen_reward": cr.mean(),
                                            "rejected_reward": rr.mean()})
