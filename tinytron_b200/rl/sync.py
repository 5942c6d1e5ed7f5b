"""Actor -> rollout weight sync (reference: tinytron/rl/sync.py:12-57).  The training
layout is resharded into the inference layout through the bridge; with a process
group each slice moves point-to-point from its owner to the rank that needs it."""
from __future__ import annotations

from dataclasses import replace

import torch

from tinytron_b200.bridge import distributed_training_state_dict_to_local_inference


def inference_model_config(model_config, shard_qkv: bool = True):
    return replace(model_config, inference_shard_qkv=shard_qkv)


def unwrap_model(model):
    return model.module if hasattr(model, "module") else model


def training_state_dict_to_inference(training_model, model_config, process_group=None):
    return distributed_training_state_dict_to_local_inference(unwrap_model(training_model).state_dict(),
                                                              model_config=model_config, process_group=process_group)


class ActorRolloutBridge:
    def __init__(self, actor_model, rollout_model, rollout_model_config, process_group=None):
        self.actor_model = actor_model
        self.rollout_model = rollout_model
        self.rollout_model_config = rollout_model_config
        self.process_group = process_group

    @torch.no_grad()
    def sync(self, strict: bool = True):
        sd = training_state_dict_to_inference(self.actor_model, self.rollout_model_config, self.process_group)
        unwrap_model(self.rollout_model).load_state_dict(sd, strict=strict)
        return sd
