"""``--preset NAME`` for the launchers: expands a named model preset
(:mod:`tinytron_b200.models.presets`) into the model flags the parsers understand.
Explicit flags given after it still win (argparse keeps the last value)."""
from __future__ import annotations

import sys

_FIELDS = (("num_layer", "num_layer"), ("num_attention_heads", "num_attention_heads"),
           ("num_key_value_heads", "num_key_value_heads"), ("hidden_size", "hidden_size"),
           ("intermediate_size", "intermediate_size"), ("vocab_size", "vocab_size"), ("block_size", "block_size"),
           ("num_experts", "num_experts"), ("num_experts_per_tok", "num_experts_per_tok"),
           ("moe_intermediate_size", "moe_intermediate_size"))


def preset_flags(name: str) -> list[str]:
    from tinytron_b200.models.presets import get_preset

    cfg = get_preset(name)
    out = []
    for attr, flag in _FIELDS:
        out += [f"--{flag}", str(getattr(cfg, attr))]
    if cfg.use_moe:
        out.append("--use_moe")
    return out


def expand_preset(argv: list[str] | None = None) -> list[str]:
    """Replace ``--preset NAME`` (or ``--preset=NAME``) in argv by the preset's flags, placed first."""
    argv = list(sys.argv[1:] if argv is None else argv)
    rest, flags = [], []
    i = 0
    while i < len(argv):
        a = argv[i]
        if a == "--preset" and i + 1 < len(argv):
            flags = preset_flags(argv[i + 1])
            i += 2
            continue
        if a.startswith("--preset="):
            flags = preset_flags(a.split("=", 1)[1])
            i += 1
            continue
        rest.append(a)
        i += 1
    return flags + rest
