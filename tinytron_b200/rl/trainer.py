"""Synchronous RL trainer (reference: tinytron/rl/trainer.py:20-222): each step syncs
the actor into the rollout engine, samples ``group_size`` completions per prompt,
scores them with a rule reward, normalises advantages within each group, recomputes
the actor's log-probs on this rank's sequence shard and applies the GRPO loss."""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist

from tinytron_b200.inference import InferenceEngine
from tinytron_b200.training.trainer import Trainer

from .logprobs import gather_log_probs
from .losses import grpo_loss
from .rollout import group_advantages, make_rollout_batch
from .sync import ActorRolloutBridge, inference_model_config


@dataclass(frozen=True)
class RLConfig:
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
    def __init__(self, config, rl_config: RLConfig):
        self.rl_config = rl_config
        super().__init__(config)
        self._init_rollout_model(config, rl_config)

    def _init_rollout_model(self, config, rl_config):
        cfg = inference_model_config(config.model, shard_qkv=rl_config.rollout_shard_qkv)
        self.rollout_engine = InferenceEngine(cfg, checkpoint_path=None, device=str(self.device),
                                              dtype=torch.bfloat16 if config.train.precision == "bf16" else torch.float32,
                                              use_paged_kv_cache=True)
        self.rollout_bridge = ActorRolloutBridge(self.raw_model, self.rollout_engine.model, cfg)

    def _one_training_step(self, config, step: int):
        self.model.train()
        self.flat.zero_grad()
        self.rollout_bridge.sync()
        dev = self.device
        ga = self.training_info["grad_accum_steps"]
        loss_acc = torch.zeros((), device=dev)
        reward_acc = torch.zeros((), device=dev)
        kl_acc = torch.zeros((), device=dev)
        tok_acc = torch.zeros((), device=dev, dtype=torch.long)
        for _ in range(ga):
            loss, m = self._one_rl_micro_step(self._next_train_batch())
            (loss / ga).backward()
            loss_acc += m["loss"] / ga
            reward_acc += m["reward"] / ga
            kl_acc += m.get("kl", torch.zeros((), device=dev)) / ga
            tok_acc += m["valid_tokens"]
        norm, coef = self._sync_and_clip(config.train.grad_clip_value)
        lr = self._lr_scheduler(step, self.training_info["max_steps"], config.optim.warmup_steps, config.optim.max_lr,
                                config.optim.min_lr)
        if self.use_flat_optimizer:
            self.optimizer.step(lr=lr, grad_scale=coef)
        else:
            for g in self.optimizer.param_groups:
                g["lr"] = lr
            self.optimizer.step()
        for t in (loss_acc, reward_acc, kl_acc):
            if self.dp_world_size > 1:
                dist.all_reduce(t, group=self.dp_group)
                t /= self.dp_world_size
        if self.dp_sp_world_size > 1:
            dist.all_reduce(tok_acc, group=self.dp_sp_group)
        self.one_step_results.update(lr=lr, loss=loss_acc, reward=reward_acc, kl=kl_acc, grad_norm=norm,
                                     valid_tokens=tok_acc)

    def _one_rl_micro_step(self, data_batch):
        prompts = data_batch["input_ids"].to(self.device).repeat_interleave(self.rl_config.group_size, dim=0)
        rollout = self._rollout(prompts)
        resp_mask = self._response_token_mask(rollout)
        rewards = self._rule_rewards(rollout.responses, resp_mask)
        adv = group_advantages(rewards, self.rl_config.group_size).to(rollout.response_mask.dtype)
        lp, old_lp, mask = self._actor_local_log_probs(rollout.sequences, rollout.labels, rollout.old_log_probs)
        loss, lm = self._policy_loss(lp, old_lp, adv, mask)
        metrics = {"loss": loss.detach(), "reward": rewards.mean().detach(), "valid_tokens": mask.sum().long()}
        metrics.update(lm)
        return loss, metrics

    def _response_token_mask(self, rollout):
        P = int(rollout.prompt_lens[0].item())
        return rollout.response_mask[:, P - 1:]

    def _rollout(self, prompts):
        self.rollout_engine.model.eval()
        seqs, info = self.rollout_engine.generate(prompts, max_new_tokens=self.rl_config.max_new_tokens,
                                                  temperature=self.rl_config.temperature, top_k=self.rl_config.top_k,
                                                  top_p=self.rl_config.top_p, eos_token_id=self.rl_config.eos_token_id,
                                                  return_logprobs=True)
        return make_rollout_batch(prompts, seqs, old_log_probs=info["token_log_probs"].detach(),
                                  eos_token_id=self.rl_config.eos_token_id)

    def _policy_loss(self, log_probs, old_log_probs, advantages, mask):
        raise NotImplementedError

    def _actor_local_log_probs(self, sequences, labels, old_log_probs):
        x_all = sequences[:, :-1]
        full_mask = labels.ne(-100).float()
        if x_all.size(1) % self.sp_world_size:
            raise ValueError("prompt_len + max_new_tokens - 1 must be divisible by sp_world_size. "
                             f"Got {x_all.size(1)} and sp_world_size={self.sp_world_size}.")
        c = x_all.size(1) // self.sp_world_size
        sl = slice(self.sp_rank * c, (self.sp_rank + 1) * c)
        x, y = x_all[:, sl].contiguous(), labels[:, sl].contiguous()
        mask, old = full_mask[:, sl].contiguous(), old_log_probs[:, sl].contiguous()
        logits = self.model(x)
        return gather_log_probs(logits, y.masked_fill(y == -100, 0)) * mask, old, mask

    def _rule_rewards(self, responses, response_mask):
        target = int(self.rl_config.reward_target_token_id)
        scale = max(int(self.config.model.vocab_size) - 1, 1)
        score = 1.0 - (responses.float() - target).abs().clamp(max=scale) / scale
        return (score * response_mask).sum(-1) / response_mask.sum(-1).clamp_min(1.0)


class GRPOTrainer(RLTrainer):
    def _policy_loss(self, log_probs, old_log_probs, advantages, mask):
        out = grpo_loss(log_probs, old_log_probs, advantages, mask, clip_range=self.rl_config.clip_range,
                        kl_coef=self.rl_config.kl_coef, group=self.sp_group)
        return out.loss, out.metrics
