"""Pretraining entry point (reference: scripts/debug/pretrain.py:16-25).

    torchrun --nproc-per-node N -m tinytron_b200.launch.pretrain [--preset NAME] [training flags]

Every flag of :func:`tinytron_b200.training.build_parser` is accepted; ``--preset``
expands a named model preset first.  Prints the reference's per-step log line
(``... | tok/sec: X | MFU: Y%``), which :mod:`tinytron_b200.launch.autotune` parses.
"""
from __future__ import annotations

from tinytron_b200.training import Trainer, build_config, parse_args

from ._presets import expand_preset


def main(argv: list[str] | None = None) -> None:
    cfg = build_config(parse_args(expand_preset(argv)))
    trainer = Trainer(cfg)
    trainer.train()


if __name__ == "__main__":
    main()
