"""Training configuration dataclasses (reference: tinytron/training/config.py:8-208).

The dataclass names, fields and defaults match the reference so configs and the
checkpoint ``meta['config']`` dict interoperate.  Extra fields (marked "ext") are
B200-specific knobs with defaults that keep reference behaviour.
"""
from __future__ import annotations

import argparse
from dataclasses import asdict, dataclass, field, replace
from typing import Any

from tinytron_b200.models.config import ModelConfig, build_model_config


@dataclass(frozen=True)
class TrainingConfig:
    total_batch_size: int = 524288  # tokens per optimizer step (global)
    batch_size: int = 8  # micro batch per device
    seq_len: int = 4096
    max_steps: int | None = None
    max_epochs: int | None = 1
    do_val: bool = False
    val_every_steps: int = 250
    split_rate: float | None = None
    grad_clip_value: float = 1.0
    debug: bool = False
    precision: str = "bf16"
    use_compile: bool = False
    use_profiler: bool = False
    steps_to_profile: list[int] = field(default_factory=lambda: [15, 20])

    def with_derived(self) -> "TrainingConfig":
        if self.split_rate is None:
            return replace(self, split_rate=0.99 if self.do_val else 1.0)
        return self


@dataclass(frozen=True)
class LoggingConfig:
    log_dir: str = "./log/"
    log_every: int = 10
    print_config: bool = False


@dataclass(frozen=True)
class SeedConfig:
    seed: int = 1337
    deterministic: bool = False


@dataclass(frozen=True)
class DataConfig:
    dataset_path: str = ""
    use_mock_data: bool = False
    mock_data_num_samples: int = 1280
    num_workers: int = 0
    pin_memory: bool = True


@dataclass(frozen=True)
class OptimConfig:
    optimizer: str = "adam"
    max_lr: float = 4e-3
    min_lr: float = 3e-5
    warmup_steps: int = 1000
    weight_decay: float = 0.1
    adam_beta1: float = 0.9
    adam_beta2: float = 0.95
    adam_eps: float = 1e-8
    muon_momentum: float = 0.95


@dataclass(frozen=True)
class CheckpointConfig:
    do_save: bool = False
    save_every_steps: int = 5000
    resume_path: str | None = None


@dataclass(frozen=True)
class ParallelConfig:
    backend: str = "nccl"
    init_method: str = "env://"
    sep_size: int = 1
    ddp_find_unused_parameters: bool = False
    ddp_gradient_as_bucket_view: bool = True
    use_distributed_optimizer: bool = True
    # ext: collective implementation of the hot paths: "native" (peer loads/stores on symmetric
    # heaps inside one node) or "nccl".
    comm_impl: str = "native"
    # ext: fp32 gradient bucket (MB) of the reduce-scatter overlapped with the backward (0: off).
    grad_bucket_mb: int = 256


@dataclass(frozen=True)
class Config:
    logging: LoggingConfig
    seed: SeedConfig
    data: DataConfig
    train: TrainingConfig
    optim: OptimConfig
    ckpt: CheckpointConfig
    parallel: ParallelConfig
    model: ModelConfig

    def as_dict(self) -> dict[str, Any]:
        return {
            "logging": asdict(self.logging),
            "seed": asdict(self.seed),
            "data": asdict(self.data),
            "train": asdict(self.train),
            "optim": asdict(self.optim),
            "ckpt": asdict(self.ckpt),
            "parallel": asdict(self.parallel),
            "model": asdict(self.model),
        }


def build_config(args: argparse.Namespace) -> Config:
    def pick(cls, **names):
        return cls(**{k: getattr(args, v) for k, v in names.items() if hasattr(args, v)})

    logging_cfg = LoggingConfig(log_dir=args.log_dir, log_every=args.log_every,
                                print_config=getattr(args, "print_config", False))
    seed_cfg = SeedConfig(seed=args.seed, deterministic=args.deterministic)
    data_cfg = DataConfig(dataset_path=args.dataset_path, use_mock_data=args.use_mock_data,
                          mock_data_num_samples=args.mock_data_num_samples, num_workers=args.num_workers,
                          pin_memory=args.pin_memory)
    train_cfg = TrainingConfig(
        total_batch_size=args.total_batch_size, batch_size=args.batch_size, seq_len=args.seq_len,
        max_steps=args.max_steps, max_epochs=args.max_epochs, do_val=args.do_val,
        val_every_steps=args.val_every_steps, split_rate=args.split_rate, grad_clip_value=args.grad_clip_value,
        debug=args.debug, precision=args.precision, use_compile=args.use_compile, use_profiler=args.use_profiler,
        steps_to_profile=list(args.steps_to_profile),
    ).with_derived()
    optim_cfg = OptimConfig(
        optimizer=args.optimizer, max_lr=args.max_lr, min_lr=args.min_lr, warmup_steps=args.warmup_steps,
        weight_decay=args.weight_decay, adam_beta1=args.adam_beta1, adam_beta2=args.adam_beta2,
        adam_eps=args.adam_eps, muon_momentum=args.muon_momentum,
    )
    ckpt_cfg = CheckpointConfig(do_save=args.do_save, save_every_steps=args.save_every_steps,
                                resume_path=args.resume_path)
    parallel_cfg = ParallelConfig(
        backend=args.backend, init_method=args.init_method, sep_size=args.sep_size,
        ddp_find_unused_parameters=args.ddp_find_unused_parameters,
        ddp_gradient_as_bucket_view=args.ddp_gradient_as_bucket_view,
        use_distributed_optimizer=args.use_distributed_optimizer,
        comm_impl=getattr(args, "comm_impl", "native"), grad_bucket_mb=getattr(args, "grad_bucket_mb", 256),
    )
    model_cfg = build_model_config(args, seed=args.seed)
    cfg = Config(logging=logging_cfg, seed=seed_cfg, data=data_cfg, train=train_cfg, optim=optim_cfg,
                 ckpt=ckpt_cfg, parallel=parallel_cfg, model=model_cfg)
    validate_static(cfg)
    return cfg


def validate_static(cfg: Config) -> None:
    """Static sanity checks; world-size dependent checks happen after dist init."""
    t, m = cfg.train, cfg.model
    if t.seq_len <= 0:
        raise ValueError("T must be positive.")
    if t.batch_size <= 0:
        raise ValueError("micro batch size B must be positive.")
    if t.total_batch_size <= 0:
        raise ValueError("total_batch_size must be positive (tokens).")
    if cfg.parallel.sep_size <= 0:
        raise ValueError("sep_size must be positive.")
    if t.precision not in ("bf16", "fp16", "fp32"):
        raise ValueError(f"Unsupported precision: {t.precision}")
    if cfg.optim.optimizer not in ("adam", "muon"):
        raise ValueError(f"Unsupported optimizer: {cfg.optim.optimizer}")
    if t.max_steps is not None and cfg.optim.warmup_steps >= t.max_steps:
        raise ValueError("warmup_steps must be < max_steps when max_steps is set.")
    if m.hidden_size % m.num_attention_heads != 0:
        raise ValueError("hidden_size must be divisible by num_attention_heads.")
    if m.num_attention_heads % m.num_key_value_heads != 0:
        raise ValueError("num_attention_heads must be divisible by num_key_value_heads (GQA).")
    if m.use_moe and m.num_experts_per_tok <= 0:
        raise ValueError("num_experts_per_tok must be positive when use_moe is enabled.")
    if m.moe_balance_loss_weight < 0:
        raise ValueError("moe_balance_loss_weight must be non-negative.")
    if cfg.parallel.comm_impl not in ("native", "nccl"):
        raise ValueError(f"Unsupported comm_impl: {cfg.parallel.comm_impl}")
