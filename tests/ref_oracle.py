"""Helpers that run the unmodified reference (installed under baseline/_ref) on CPU
as a numerical oracle.  The reference hard-codes CUDA devices; two torch-level
patches make it build on CPU: torch.cuda.current_device -> "cpu" and fork_rng
restricted to the CPU generator.  No reference source is modified."""
from __future__ import annotations

import contextlib
import os
import sys

import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_DIR = os.path.join(ROOT, "baseline", "_ref")


def available() -> bool:
    return os.path.isdir(os.path.join(REF_DIR, "tinytron"))


@contextlib.contextmanager
def cpu_reference():
    """Import the reference package with CPU patches active; yields the `tinytron` module."""
    if REF_DIR not in sys.path:
        sys.path.insert(0, REF_DIR)
    orig_dev = torch.cuda.current_device
    orig_fork = torch.random.fork_rng
    torch.cuda.current_device = lambda: "cpu"
    torch.random.fork_rng = lambda devices=None, **kw: orig_fork(devices=[], **kw)
    try:
        import tinytron  # noqa: F401

        yield sys.modules["tinytron"]
    finally:
        torch.cuda.current_device = orig_dev
        torch.random.fork_rng = orig_fork


def ensure_gloo_world1(port: int = 29611):
    import torch.distributed as dist

    if not dist.is_initialized():
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=0, world_size=1)
