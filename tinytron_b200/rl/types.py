"""RL data types (reference: tinytron/rl/types.py:8-38)."""
from __future__ import annotations

from dataclasses import dataclass, fields

import torch


@dataclass
class RLLossOutput:
    loss: torch.Tensor
    metrics: dict[str, torch.Tensor]


@dataclass
class RolloutBatch:
    """labels, response_mask and the log-prob tensors are aligned to sequences[:, 1:];
    non-action labels are -100 (the training batch convention)."""

    prompts: torch.Tensor
    responses: torch.Tensor
    sequences: torch.Tensor
    labels: torch.Tensor
    response_mask: torch.Tensor
    prompt_lens: torch.Tensor
    response_lens: torch.Tensor
    old_log_probs: torch.Tensor | None = None
    reference_log_probs: torch.Tensor | None = None
    rewards: torch.Tensor | None = None
    advantages: torch.Tensor | None = None

    def to(self, device) -> "RolloutBatch":
        return RolloutBatch(**{f.name: (getattr(self, f.name).to(device) if torch.is_tensor(getattr(self, f.name))
                                        else getattr(self, f.name)) for f in fields(self)})
