"""tinytron_b200: a Blackwell-native (sm_100a) GPT/MoE pretraining and inference stack
with Tinytron's capabilities, public API and sharded-checkpoint format.

Sub-packages: ``models`` (GPT/MoE modules), ``ops`` (sm_100a kernels + autograd),
``parallel`` (process groups, DDP/ZeRO-1, Ulysses, expert parallel, peer-memory
runtime), ``optim`` (AdamW, Muon), ``training``, ``inference``, ``bridge``
(layout-aware checkpoint resharding), ``rl`` and ``utils``.

The reference's import paths ``<pkg>.model`` and ``<pkg>.distributed`` are
provided as aliases of ``models`` and ``parallel``.
"""
from __future__ import annotations

import importlib
import importlib.abc
import importlib.util
import sys

__version__ = "0.1.0"

_ALIASES = {
    "tinytron_b200.model": "tinytron_b200.models",
    "tinytron_b200.distributed": "tinytron_b200.parallel",
}


class _AliasLoader(importlib.abc.Loader):
    def __init__(self, real: str):
        self.real = real

    def create_module(self, spec):
        return importlib.import_module(self.real)

    def exec_module(self, module):
        return None


class _AliasFinder(importlib.abc.MetaPathFinder):
    def find_spec(self, fullname, path, target=None):
        for alias, real in _ALIASES.items():
            if fullname == alias or fullname.startswith(alias + "."):
                target_name = real + fullname[len(alias):]
                if importlib.util.find_spec(target_name) is None:
                    return None
                return importlib.util.spec_from_loader(fullname, _AliasLoader(target_name))
        return None


if not any(isinstance(f, _AliasFinder) for f in sys.meta_path):
    sys.meta_path.insert(0, _AliasFinder())
