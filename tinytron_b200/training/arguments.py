"""Training CLI (reference: tinytron/training/arguments.py:8-120): same flag names,
groups and defaults, plus a few B200 extensions (``--comm_impl``, ``--grad_bucket_mb``, ``--rms_norm_eps``,
``--rope_theta``, ``--model_preset``)."""
from __future__ import annotations

import argparse

from tinytron_b200.models.config import add_model_config_args


def add_all_arguments(parser: argparse.ArgumentParser) -> argparse.ArgumentParser:
    for fn in (_logging, _seed, _data, _training, _optim, _checkpoint, _parallel, _model):
        parser = fn(parser)
    return parser


def build_parser() -> argparse.ArgumentParser:
    return add_all_arguments(argparse.ArgumentParser("pretrain", allow_abbrev=False))


def parse_args(argv: list[str] | None = None) -> argparse.Namespace:
    return build_parser().parse_args(argv)


def _training(p):
    g = p.add_argument_group("training")
    g.add_argument("--total_batch_size", type=int, default=524288, help="global batch size in tokens")
    g.add_argument("--batch_size", type=int, default=8, help="micro batch size per device")
    g.add_argument("--seq_len", type=int, default=4096)
    g.add_argument("--max_steps", type=int, default=None)
    g.add_argument("--max_epochs", type=int, default=None)
    g.add_argument("--do_val", action="store_true")
    g.add_argument("--val_every_steps", type=int, default=250)
    g.add_argument("--split_rate", type=float, default=None)
    g.add_argument("--grad_clip_value", type=float, default=1.0)
    g.add_argument("--debug", action="store_true")
    g.add_argument("--precision", type=str, default="bf16", choices=["bf16", "fp16", "fp32"])
    g.add_argument("--use_compile", action="store_true", help="accepted for CLI compatibility; kernels are native")
    g.add_argument("--use_profiler", action="store_true")
    g.add_argument("--steps_to_profile", type=int, nargs="+", default=[15, 20])
    return p


def _logging(p):
    g = p.add_argument_group("logging")
    g.add_argument("--log_dir", type=str, default="./log/")
    g.add_argument("--log_every", type=int, default=10)
    g.add_argument("--print_config", action="store_true")
    return p


def _seed(p):
    g = p.add_argument_group("reproducibility")
    g.add_argument("--seed", type=int, default=1337)
    g.add_argument("--deterministic", action="store_true")
    return p


def _data(p):
    g = p.add_argument_group("data")
    g.add_argument("--dataset_path", type=str, default="../data/fineweb-edu-sample-10BT/")
    g.add_argument("--use_mock_data", action="store_true")
    g.add_argument("--mock_data_num_samples", type=int, default=1280)
    g.add_argument("--num_workers", type=int, default=0)
    g.add_argument("--pin_memory", action=argparse.BooleanOptionalAction, default=True)
    return p


def _optim(p):
    g = p.add_argument_group("optimizer")
    g.add_argument("--optimizer", type=str, default="adam")
    g.add_argument("--max_lr", type=float, default=4e-3)
    g.add_argument("--min_lr", type=float, default=3e-5)
    g.add_argument("--warmup_steps", type=int, default=1000)
    g.add_argument("--weight_decay", type=float, default=0.1)
    g.add_argument("--adam_beta1", type=float, default=0.9)
    g.add_argument("--adam_beta2", type=float, default=0.95)
    g.add_argument("--adam_eps", type=float, default=1e-8)
    g.add_argument("--muon_momentum", type=float, default=0.95)
    return p


def _checkpoint(p):
    g = p.add_argument_group("checkpoint")
    g.add_argument("--do_save", action="store_true")
    g.add_argument("--save_every_steps", type=int, default=5000)
    g.add_argument("--resume_path", type=str, default=None)
    return p


def _parallel(p):
    g = p.add_argument_group("distributed")
    g.add_argument("--backend", type=str, default="nccl")
    g.add_argument("--init_method", type=str, default="env://")
    g.add_argument("--sep_size", type=int, default=1, help="SEP size (SP/EP joint parallel group size)")
    g.add_argument("--ddp_find_unused_parameters", action="store_true")
    g.add_argument("--ddp_gradient_as_bucket_view", action=argparse.BooleanOptionalAction, default=True)
    g.add_argument("--use_distributed_optimizer", action=argparse.BooleanOptionalAction, default=True)
    g.add_argument("--grad_bucket_mb", type=int, default=256,
                   help="native ZeRO-1 (DP, no SEP): fp32 gradient bucket size whose reduce-scatter overlaps "
                        "the last micro-step's backward; 0 reduce-scatters everything after the backward")
    g.add_argument("--comm_impl", type=str, default="native", choices=["native", "nccl"],
                   help="native: ZeRO-1, EP and Ulysses collectives as NVLink peer loads/stores on symmetric "
                        "heaps (one node); nccl: every collective on NCCL")
    return p


def _model(p):
    g = p.add_argument_group("model")
    add_model_config_args(g)
    return p
