"""RL primitives and trainers (reference API: tinytron/rl/__init__.py:18-42)."""
from .logprobs import (build_response_mask, causal_log_probs, gather_log_probs, masked_mean, masked_sum,
                       response_log_probs, sequence_log_probs)
from .losses import approx_kl, dpo_loss, grpo_loss, policy_gradient_loss, ppo_policy_loss
from .rollout import group_advantages, make_rollout_batch
from .sync import ActorRolloutBridge, inference_model_config, training_state_dict_to_inference, unwrap_model
from .types import RLLossOutput, RolloutBatch

__all__ = ["RLLossOutput", "RolloutBatch", "ActorRolloutBridge", "GRPOTrainer", "RLConfig", "RLTrainer", "approx_kl",
           "build_response_mask", "causal_log_probs", "dpo_loss", "gather_log_probs", "grpo_loss", "group_advantages",
           "inference_model_config", "make_rollout_batch", "masked_mean", "masked_sum", "policy_gradient_loss",
           "ppo_policy_loss", "response_log_probs", "sequence_log_probs", "training_state_dict_to_inference",
           "unwrap_model"]


def __getattr__(name):
    if name in ("GRPOTrainer", "RLConfig", "RLTrainer"):
        from . import trainer

        return getattr(trainer, name)
    raise AttributeError(name)
