"""Model package (reference API: tinytron/model/__init__.py:5-41)."""
from __future__ import annotations

from .config import ModelConfig, add_model_config_args, build_model_config

__all__ = ["ModelConfig", "add_model_config_args", "build_model_config", "GPT", "Block", "TextEmbedding",
           "ImgEmbedding", "Attention", "MLP", "MoE", "LayerNorm"]


def __getattr__(name: str):
    if name in {"GPT", "Block"}:
        from . import gpt

        return getattr(gpt, name)
    if name in {"TextEmbedding", "ImgEmbedding"}:
        from .modules import emb

        return getattr(emb, name)
    if name == "Attention":
        from .modules.attn import Attention

        return Attention
    if name in {"MLP", "MoE"}:
        from .modules import mlp

        return getattr(mlp, name)
    if name == "LayerNorm":
        from .modules.norm import LayerNorm

        return LayerNorm
    raise AttributeError(f"module {__name__!r} has no attribute {name!r}")
