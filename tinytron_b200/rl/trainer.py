"""Synchronous on-policy RL trainers (capabilities of the reference's
tinytron/rl/trainer.py:20-222: ``RLConfig``, ``RLTrainer``, ``GRPOTrainer``).

One optimizer step runs in two phases:

1. Rollout.  The actor's weights are synced into the inference engine (through the
   resharding bridge), then the prompts of ALL gradient-accumulation micro-batches,
   each repeated ``group_size`` times, are generated in ONE batched ``generate`` call:
   ``grad_accum`` times more sequences share every decode step (and its CUDA graph)
   than with one rollout per micro-batch, which is what keeps a B200 busy at decode.
   The actor does not change during a step, so this samples from the same policy.
2. Learn.  For each micro-batch: rule rewards and group-normalised advantages, the
   actor's per-token log-probs on this rank's sequence shard (through the fused
   LM-head + cross-entropy kernel, ``GPT.token_log_probs``: no ``[B, T, V]`` fp32
   log-softmax), the policy loss and its backward into the flat fp32 gradients.

The gradient sync, clipping and update reuse the pretraining trainer's path (flat
ZeRO-1 AdamW, or Muon); the step's scalar metrics cross ranks in one packed
all-reduce.  Subclasses supply ``_policy_loss``; ``_rule_rewards`` and ``_rollout``
are the other extension points.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist

from tinytron_b200.inference import InferenceEngine
from tinytron_b200.training.trainer import Trainer

from .logprobs import packed_all_reduce
from .losses import grpo_loss
from .rollout import group_advantages, make_rollout_batch
from .sync import ActorRolloutBridge, inference_model_config
from .types import RolloutBatch


@dataclass(frozen=True)
class RLConfig:
    """Rollout and objective settings (field names and defaults are the reference's)."""

    max_new_tokens: int = 8
    group_size: int = 2
    temperature: float = 1.0
    top_k: int | None = None
    top_p: float | None = None
    eos_token_id: int | None = None
    reward_target_token_id: int = 0
    clip_range: float = 0.2
    kl_coef: float = 0.0
    rollout_shard_qkv: bool = True


class RLTrainer(Trainer):
    """Base trainer: batched rollout, then per-micro-batch policy-gradient updates."""

    def __init__(self, config, rl_config: RLConfig):
        self.rl_config = rl_config
        super().__init__(config)
        self._init_rollout_model(config, rl_config)

    def _init_rollout_model(self, config, rl_config: RLConfig) -> None:
        cfg = inference_model_config(config.model, shard_qkv=rl_config.rollout_shard_qkv)
        dtype = torch.bfloat16 if config.train.precision == "bf16" else torch.float32
        self.rollout_engine = InferenceEngine(cfg, checkpoint_path=None, device=str(self.device), dtype=dtype,
                                              use_paged_kv_cache=True)
        self.rollout_bridge = ActorRolloutBridge(self.raw_model, self.rollout_engine.model, cfg)

    # ------------------------------------------------------------------ one optimizer step
    def _one_training_step(self, config, step: int):
        self.model.train()
        self.flat.zero_grad()
        self.rollout_bridge.sync()
        ga = self.training_info["grad_accum_steps"]
        batches = self._rollout_all([self._next_train_batch() for _ in range(ga)])
        zero = torch.zeros((), device=self.device)
        loss_sum, reward_sum, kl_sum = zero.clone(), zero.clone(), zero.clone()
        tokens = torch.zeros((), device=self.device, dtype=torch.long)
        for rollout in batches:
            loss, m = self._learn_on(rollout)
            (loss / ga).backward()
            loss_sum += m["loss"]
            reward_sum += m["reward"]
            kl_sum += m.get("kl", zero)
            tokens += m["valid_tokens"]
        norm, coef = self._sync_and_clip(config.train.grad_clip_value)
        lr = self._lr_scheduler(step, self.training_info["max_steps"], config.optim.warmup_steps,
                                config.optim.max_lr, config.optim.min_lr)
        if self.use_flat_optimizer:
            self.optimizer.step(lr=lr, grad_scale=coef)
        else:
            for g in self.optimizer.param_groups:
                g["lr"] = lr
            self.optimizer.step(grad_scale=coef)
            for p in self.flat.params:
                p.grad = None
            if self.device.type == "cuda":
                self.flat.refresh_bf16()
        # DP means of the per-micro-batch averages, and the global valid-token count: one
        # collective for the three float metrics (the token count is summed over DP x SP).
        means = torch.stack([loss_sum, reward_sum, kl_sum]) / ga
        if self.dp_world_size > 1:
            (means,) = packed_all_reduce([means], self.dp_group)
            means = means / self.dp_world_size
        if self.dp_sp_world_size > 1:
            dist.all_reduce(tokens, group=self.dp_sp_group)
        self.one_step_results.update(lr=lr, loss=means[0], reward=means[1], kl=means[2], grad_norm=norm,
                                     valid_tokens=tokens)

    # ------------------------------------------------------------------ rollout phase
    def _rollout_all(self, data_batches: list[dict]) -> list[RolloutBatch]:
        """Generate completions for every micro-batch's prompts in one engine call and
        split the result back into per-micro-batch rollout batches."""
        prompts = [b["input_ids"].to(self.device).repeat_interleave(self.rl_config.group_size, dim=0)
                   for b in data_batches]
        if len({p.shape[1] for p in prompts}) != 1:  # mixed prompt lengths: one call per micro-batch
            return [self._rollout(p) for p in prompts]
        full = self._rollout(torch.cat(prompts, 0))
        out, r0 = [], 0
        for p in prompts:
            r1 = r0 + p.shape[0]
            out.append(RolloutBatch(**{k: (v[r0:r1] if torch.is_tensor(v) else v) for k, v in vars(full).items()}))
            r0 = r1
        return out

    def _rollout(self, prompts: torch.Tensor) -> RolloutBatch:
        self.rollout_engine.model.eval()
        rc = self.rl_config
        sequences, info = self.rollout_engine.generate(prompts, max_new_tokens=rc.max_new_tokens,
                                                       temperature=rc.temperature, top_k=rc.top_k, top_p=rc.top_p,
                                                       eos_token_id=rc.eos_token_id, return_logprobs=True)
        return make_rollout_batch(prompts, sequences, old_log_probs=info["token_log_probs"].detach(),
                                  eos_token_id=rc.eos_token_id)

    # ------------------------------------------------------------------ learn phase
    def _learn_on(self, rollout: RolloutBatch):
        P = rollout.prompts.shape[1]
        generated_mask = rollout.response_mask[:, P - 1:]
        rewards = self._rule_rewards(rollout.responses, generated_mask)
        advantages = group_advantages(rewards, self.rl_config.group_size).to(rollout.response_mask.dtype)
        log_probs, old_log_probs, mask = self._actor_local_log_probs(rollout.sequences, rollout.labels,
                                                                      rollout.old_log_probs)
        loss, metrics = self._policy_loss(log_probs, old_log_probs, advantages, mask)
        out = {"loss": loss.detach(), "reward": rewards.mean().detach(), "valid_tokens": mask.sum().long()}
        out.update(metrics)
        return loss, out

    def _sequence_shard(self, width: int) -> slice:
        if width % self.sp_world_size:
            raise ValueError(f"the trained sequence length prompt_len + max_new_tokens - 1 = {width} must be "
                             f"divisible by the SEP size {self.sp_world_size}")
        c = width // self.sp_world_size
        return slice(self.sp_rank * c, (self.sp_rank + 1) * c)

    def _actor_local_log_probs(self, sequences, labels, old_log_probs):
        """(log-probs, sampler log-probs, mask) of this rank's contiguous sequence shard;
        non-action positions (label -100) carry log-prob 0 and mask 0."""
        inputs = sequences[:, :-1]
        sl = self._sequence_shard(inputs.shape[1])
        x = inputs[:, sl].contiguous()
        y = labels[:, sl].contiguous()
        mask = y.ne(-100).to(torch.float32)
        log_probs = self.raw_model.token_log_probs(x, y)
        return log_probs * mask, old_log_probs[:, sl].contiguous(), mask

    def _rule_rewards(self, responses: torch.Tensor, response_mask: torch.Tensor) -> torch.Tensor:
        """Toy verifiable reward: per generated token, 1 - |token - target| / (V - 1),
        averaged over each response's valid tokens (the reference's rule reward)."""
        target = float(self.rl_config.reward_target_token_id)
        span = float(max(int(self.config.model.vocab_size) - 1, 1))
        closeness = 1.0 - (responses.float() - target).abs().clamp(max=span) / span
        m = response_mask.to(closeness.dtype)
        return (closeness * m).sum(-1) / m.sum(-1).clamp_min(1.0)

    def _policy_loss(self, log_probs, old_log_probs, advantages, mask):
        raise NotImplementedError("RLTrainer subclasses define the policy objective")


class GRPOTrainer(RLTrainer):
    """Group-relative policy optimisation: the PPO clipped surrogate on group-normalised
    advantages, optionally with a KL penalty; statistics reduced over the SEP group."""

    def _policy_loss(self, log_probs, old_log_probs, advantages, mask):
        out = grpo_loss(log_probs, old_log_probs, advantages, mask, clip_range=self.rl_config.clip_range,
                        kl_coef=self.rl_config.kl_coef, group=self.sp_group)
        return out.loss, out.metrics
