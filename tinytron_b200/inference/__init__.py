"""Inference (reference API: tinytron/inference/__init__.py:1-4)."""
from .engine import InferenceEngine
from .sampler import filter_logits, sample_next_token, sample_next_token_with_log_prob

__all__ = ["InferenceEngine", "filter_logits", "sample_next_token", "sample_next_token_with_log_prob"]
