"""Optimizers (reference API: tinytron/optim/__init__.py): ``AdamW`` (torch's, for
user code; the trainer's fast path is the fused flat ZeRO-1 AdamW kernel) and
``Muon`` (Newton-Schulz orthogonalised momentum with an Adam branch)."""
from torch.optim import AdamW

from .muon import Muon, adam_update, muon_update, zeropower_via_newtonschulz5

__all__ = ["AdamW", "Muon", "zeropower_via_newtonschulz5", "muon_update", "adam_update"]
