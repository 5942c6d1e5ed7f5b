"""Model configuration (reference: tinytron/model/config.py:7-71).

Same frozen dataclass fields and CLI flags as the reference, plus two knobs the
reference hard-codes: ``rms_norm_eps`` (reference fixes 1e-6, norm.py:10) and
``rope_theta`` (reference fixes 10000, attn.py:17).  Defaults keep the
reference's values so checkpoints and numerics line up.
"""
from __future__ import annotations

import argparse
from dataclasses import dataclass


@dataclass(frozen=True)
class ModelConfig:
    seed: int = 1337
    block_size: int = 4096
    vocab_size: int = 50304
    num_layer: int = 32
    num_attention_heads: int = 128
    num_key_value_heads: int = 8
    hidden_size: int = 1024
    intermediate_size: int = 4096
    dropout: float = 0.0
    init_std: float = 0.013
    tied_lm_head: bool = True

    # MoE
    use_moe: bool = False
    num_experts: int = 128
    num_experts_per_tok: int = 8
    moe_intermediate_size: int = 256
    moe_balance_loss_weight: float = 0.01

    # Inference-only: shard q/k/v projections by SEP head shard.
    inference_shard_qkv: bool = False

    # Knobs fixed in the reference.
    rms_norm_eps: float = 1e-6
    rope_theta: float = 10000.0

    @property
    def head_dim(self) -> int:
        return self.hidden_size // self.num_attention_heads


def add_model_config_args(parser):
    d = ModelConfig()
    parser.add_argument("--block_size", type=int, default=d.block_size)
    parser.add_argument("--vocab_size", type=int, default=d.vocab_size)
    parser.add_argument("--num_layer", type=int, default=d.num_layer)
    parser.add_argument("--num_attention_heads", type=int, default=d.num_attention_heads)
    parser.add_argument("--num_key_value_heads", type=int, default=d.num_key_value_heads)
    parser.add_argument("--hidden_size", type=int, default=d.hidden_size)
    parser.add_argument("--intermediate_size", type=int, default=d.intermediate_size)
    parser.add_argument("--dropout", type=float, default=d.dropout)
    parser.add_argument("--init_std", type=float, default=d.init_std)
    parser.add_argument("--tied_lm_head", action=argparse.BooleanOptionalAction, default=d.tied_lm_head)
    parser.add_argument("--use_moe", action="store_true")
    parser.add_argument("--num_experts", type=int, default=d.num_experts)
    parser.add_argument("--num_experts_per_tok", type=int, default=d.num_experts_per_tok)
    parser.add_argument("--moe_intermediate_size", type=int, default=d.moe_intermediate_size)
    parser.add_argument("--moe_balance_loss_weight", type=float, default=d.moe_balance_loss_weight)
    parser.add_argument("--rms_norm_eps", type=float, default=d.rms_norm_eps)
    parser.add_argument("--rope_theta", type=float, default=d.rope_theta)
    parser.add_argument("--model_preset", type=str, default=None,
                        help="named preset (see tinytron_b200.models.presets); explicit flags are ignored when set")
    return parser


_FIELDS = (
    "block_size", "vocab_size", "num_layer", "num_attention_heads", "num_key_value_heads", "hidden_size",
    "intermediate_size", "dropout", "init_std", "tied_lm_head", "use_moe", "num_experts", "num_experts_per_tok",
    "moe_intermediate_size", "moe_balance_loss_weight", "rms_norm_eps", "rope_theta",
)


def build_model_config(args: argparse.Namespace, **overrides) -> ModelConfig:
    preset = getattr(args, "model_preset", None)
    if preset:
        from .presets import get_preset

        values = dict(get_preset(preset).__dict__)
        values.pop("seed", None)
    else:
        values = {f: getattr(args, f) for f in _FIELDS if hasattr(args, f)}
    values.update(overrides)
    return ModelConfig(**values)
