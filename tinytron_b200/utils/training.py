"""Schedule math and seeding (reference: tinytron/utils/training.py:10-82)."""
from __future__ import annotations

import random
from typing import Any

import numpy as np
import torch


def get_training_info(num_samples: int, tokens_per_sample: int, global_token_batch_size: int,
                      samples_per_dp_rank_per_micro_step: int, dp_world_size: int, max_steps=None,
                      max_epochs=None) -> dict[str, Any]:
    """Gradient-accumulation steps and step/epoch budget; raises if both budgets are
    given and disagree (same rule as the reference)."""
    if max_steps is None and max_epochs is None:
        raise ValueError("At least one of max_steps or max_epochs must be provided.")
    per_micro = tokens_per_sample * samples_per_dp_rank_per_micro_step * dp_world_size
    grad_accum = int(global_token_batch_size / per_micro)
    dataset_tokens = num_samples * tokens_per_sample
    if max_steps is not None and max_epochs is not None:
        calc_steps = int((max_epochs * dataset_tokens) / global_token_batch_size)
        calc_epochs = (max_steps * global_token_batch_size) / dataset_tokens
        if not (calc_steps == max_steps and int(calc_epochs) == int(max_epochs)):
            raise ValueError(
                "Inconsistent max_steps and max_epochs based on the dataset and configuration. "
                f"Calculated max_steps from max_epochs: {calc_steps}, provided max_steps: {max_steps}. "
                f"Calculated max_epochs from max_steps: {int(calc_epochs)}, provided max_epochs: {max_epochs}.")
    elif max_steps is None:
        max_steps = int((max_epochs * dataset_tokens) / global_token_batch_size)
    else:
        max_epochs = (max_steps * global_token_batch_size) / dataset_tokens
    return {"epochs": max_epochs, "max_steps": max_steps, "grad_accum_steps": grad_accum,
            "total_tokens_per_micro_step": per_micro}


def set_seed(seed: int, deterministic: bool = False) -> None:
    random.seed(seed)
    np.random.seed(seed)
    torch.manual_seed(seed)
    torch.cuda.manual_seed_all(seed)
    if deterministic:
        torch.use_deterministic_algorithms(True, warn_only=True)
        # Deterministic mode would also fill every torch.empty() with NaN (a full write of
        # each allocation, ~2 GB per step here).  No kernel of this framework reads memory it
        # has not written, so the fill only costs bandwidth.
        torch.utils.deterministic.fill_uninitialized_memory = False
