"""Training package (reference API: tinytron/training/__init__.py:6-19)."""
from .arguments import build_parser, parse_args
from .config import build_config

__all__ = ["build_parser", "parse_args", "build_config", "Trainer"]


def __getattr__(name):
    if name == "Trainer":
        from .trainer import Trainer

        return Trainer
    raise AttributeError(name)
