"""GRPO entry point (reference: scripts/debug/rl.py:14-55): training flags plus the
``--rl_*`` group; the reward is the reference's mock reward (tokens close to
``--rl_reward_target_token_id``)."""
from __future__ import annotations

import argparse

from tinytron_b200.rl import GRPOTrainer, RLConfig
from tinytron_b200.training import build_config
from tinytron_b200.training.arguments import add_all_arguments

from ._presets import expand_preset


def add_rl_args(parser: argparse.ArgumentParser) -> argparse.ArgumentParser:
    g = parser.add_argument_group("rl")
    g.add_argument("--rl_max_new_tokens", type=int, default=8)
    g.add_argument("--rl_group_size", type=int, default=2)
    g.add_argument("--rl_temperature", type=float, default=1.0)
    g.add_argument("--rl_top_k", type=int, default=0, help="0 disables top-k filtering")
    g.add_argument("--rl_top_p", type=float, default=0.0, help="0 disables top-p filtering")
    g.add_argument("--rl_eos_token_id", type=int, default=None)
    g.add_argument("--rl_reward_target_token_id", type=int, default=0)
    g.add_argument("--rl_clip_range", type=float, default=0.2)
    g.add_argument("--rl_kl_coef", type=float, default=0.0)
    g.add_argument("--rl_rollout_shard_qkv", action="store_true")
    return parser


def build_rl_config(args) -> RLConfig:
    return RLConfig(max_new_tokens=args.rl_max_new_tokens, group_size=args.rl_group_size,
                    temperature=args.rl_temperature, top_k=args.rl_top_k or None, top_p=args.rl_top_p or None,
                    eos_token_id=args.rl_eos_token_id, reward_target_token_id=args.rl_reward_target_token_id,
                    clip_range=args.rl_clip_range, kl_coef=args.rl_kl_coef,
                    rollout_shard_qkv=args.rl_rollout_shard_qkv)


def main(argv: list[str] | None = None) -> None:
    parser = add_rl_args(add_all_arguments(argparse.ArgumentParser("rl", allow_abbrev=False)))
    args = parser.parse_args(expand_preset(argv))
    trainer = GRPOTrainer(build_config(args), build_rl_config(args))
    trainer.train()


if __name__ == "__main__":
    main()
