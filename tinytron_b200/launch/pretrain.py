"""Pretraining entry point (reference: scripts/debug/pretrain.py:16-25).

    torchrun --nproc-per-node N -m tinytron_b200.launch.pretrain [--preset NAME] [training flags]

Every flag of :func:`tinytron_b200.training.build_parser` is accepted; ``--preset``
expands a named model preset first.  Prints the reference's per-step log line
(``... | tok/sec: X | MFU: Y%``), which :mod:`tinytron_b200.launch.autotune` parses.

``--streaming_data_dir DIR`` trains on token shards (``DIR/meta.json`` + ``chunk_*.bin``,
see :mod:`tinytron_b200.training.streaming`) instead of mock data, with the dataset
position saved in checkpoints (the reference's example entry point,
scripts/example/pretrain.py:76-294); ``--streaming_shuffle`` permutes samples per epoch.
"""
from __future__ import annotations

import argparse
from dataclasses import replace

from tinytron_b200.training import Trainer, build_config, parse_args

from ._presets import expand_preset


def main(argv: list[str] | None = None) -> None:
    extra = argparse.ArgumentParser(add_help=False)
    extra.add_argument("--streaming_data_dir", type=str, default=None)
    extra.add_argument("--streaming_shuffle", action="store_true")
    known, rest = extra.parse_known_args(expand_preset(argv))
    cfg = build_config(parse_args(rest))
    if known.streaming_data_dir:
        from tinytron_b200.training.streaming import StreamingTrainer

        cfg = replace(cfg, data=replace(cfg.data, dataset_path=known.streaming_data_dir, use_mock_data=False))
        StreamingTrainer.streaming_shuffle = known.streaming_shuffle
        trainer = StreamingTrainer(cfg)
    else:
        trainer = Trainer(cfg)
    trainer.train()


if __name__ == "__main__":
    main()
