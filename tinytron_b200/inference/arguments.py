"""Inference CLI (reference: tinytron/inference/arguments.py:8-70): same flags."""
from __future__ import annotations

import argparse

from tinytron_b200.models.config import add_model_config_args


def parse_prompt_token_ids(prompt: str) -> list[int]:
    vals = [p.strip() for p in prompt.split(",") if p.strip()]
    if not vals:
        raise ValueError("--prompt_token_ids must contain at least one token id")
    return [int(v) for v in vals]


def add_all_arguments(parser: argparse.ArgumentParser) -> argparse.ArgumentParser:
    g = parser.add_argument_group("inference")
    g.add_argument("--checkpoint_path", type=str, default=None, help="Path to *_model.pt checkpoint")
    g.add_argument("--init_from_scratch", action="store_true", help="Run inference with random initialized weights")
    g.add_argument("--prompt_token_ids", type=str, required=True, help="Comma-separated token ids, e.g. '1,2,3'")
    g.add_argument("--max_new_tokens", type=int, default=64)
    g.add_argument("--device", type=str, default="cuda")
    g.add_argument("--dtype", type=str, default="bf16", choices=["bf16", "fp32"])
    g.add_argument("--paged_kv_cache", action=argparse.BooleanOptionalAction, default=True)
    g.add_argument("--kv_cache_page_size", type=int, default=128)
    g = parser.add_argument_group("sampling")
    g.add_argument("--temperature", type=float, default=1.0)
    g.add_argument("--top_k", type=int, default=None)
    g.add_argument("--top_p", type=float, default=None)
    g.add_argument("--eos_token_id", type=int, default=None)
    g = parser.add_argument_group("distributed")
    g.add_argument("--backend", type=str, default="nccl")
    g.add_argument("--init_method", type=str, default="env://")
    g.add_argument("--sep_size", type=int, default=1, help="SEP size for distributed KV-cache inference")
    g = parser.add_argument_group("model")
    g.add_argument("--seed", type=int, default=1337)
    add_model_config_args(g)
    g.add_argument("--inference_shard_qkv", action=argparse.BooleanOptionalAction, default=None)
    return parser


def build_parser() -> argparse.ArgumentParser:
    return add_all_arguments(argparse.ArgumentParser("tinytron-inference", allow_abbrev=False))


def parse_args(argv=None) -> argparse.Namespace:
    return build_parser().parse_args(argv)
