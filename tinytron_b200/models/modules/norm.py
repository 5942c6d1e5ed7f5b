"""RMSNorm, named ``LayerNorm`` as in the reference (tinytron/model/modules/norm.py:6-19).

fp32 math, no bias, weight initialised to ones; eps comes from
``ModelConfig.rms_norm_eps`` (reference fixes 1e-6).  On CUDA the norm is fused
with the preceding residual add and emits the bf16 projection input directly.
"""
from __future__ import annotations

import torch
import torch.nn as nn

from tinytron_b200 import ops


def default_device():
    return torch.device("cuda", torch.cuda.current_device()) if torch.cuda.is_available() else torch.device("cpu")


class LayerNorm(nn.Module):
    def __init__(self, config, device=None):
        super().__init__()
        device = device if device is not None else default_device()
        self.variance_epsilon = float(getattr(config, "rms_norm_eps", 1e-6))
        self.hidden_size = config.hidden_size
        self.weight = nn.Parameter(torch.ones(self.hidden_size, device=device))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return ops.rmsnorm(x, self.weight, self.variance_epsilon)
