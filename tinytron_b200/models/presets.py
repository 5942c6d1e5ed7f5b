"""Named model presets.

The reference keeps these only in shell launchers
(scripts/debug/pretrain.sh:96-321, scripts/debug/inference.sh:63-179); here they
are a Python table the launchers, the benchmark and tests share.  All use
block_size 4096, vocab 50304, tied LM head, dropout 0.  The ``b200-*`` entries are
the benchmark configurations (dense 1.3B, MoE 64x1408 top-8, long-context).
"""
from __future__ import annotations

from dataclasses import replace

from .config import ModelConfig

_BASE = ModelConfig(block_size=4096, vocab_size=50304, tied_lm_head=True, dropout=0.0)


def _d(L, hq, hkv, d, i):
    return replace(_BASE, num_layer=L, num_attention_heads=hq, num_key_value_heads=hkv, hidden_size=d,
                   intermediate_size=i)


def _m(L, hq, hkv, d, i, e, k, im):
    return replace(_d(L, hq, hkv, d, i), use_moe=True, num_experts=e, num_experts_per_tok=k,
                   moe_intermediate_size=im)


PRESETS: dict[str, ModelConfig] = {
    "0.03B": _d(6, 8, 2, 512, 2048),
    "0.1B": _d(12, 16, 4, 768, 3072),
    "0.25B": _d(12, 32, 4, 1024, 4096),
    "1B": _d(24, 64, 8, 2048, 8192),
    "1.3B": _d(24, 16, 8, 2048, 6144),
    "7B": _d(32, 128, 16, 4096, 16384),
    "13B": _d(40, 40, 8, 5120, 13824),
    "30B": _d(60, 52, 8, 6656, 17920),
    "70B": _d(80, 64, 8, 8192, 28672),
    "0.17B-A0.1B": _m(12, 16, 4, 768, 3072, 8, 2, 768),
    "0.3B-A0.17B": _m(12, 32, 4, 768, 3072, 8, 2, 768),
    "0.7B-A0.25B": _m(24, 32, 4, 1024, 4096, 8, 2, 1024),
    "2.7B-A1B": _m(24, 64, 8, 2048, 8192, 8, 2, 2048),
    "14B-A4.5B": _m(32, 128, 16, 4096, 16384, 8, 2, 4096),
    "104B-A4.5B": _m(32, 128, 16, 4096, 16384, 64, 2, 4096),
    # Benchmark configurations.
    "b200-tiny-cpu": replace(_d(4, 8, 2, 256, 688), vocab_size=8192, block_size=256, init_std=0.02),
    "b200-dense-1.3b": replace(_d(24, 16, 4, 2048, 5504), init_std=0.02),
    "b200-moe-16x64": replace(_m(16, 16, 4, 2048, 5504, 64, 8, 1408), init_std=0.02),
    "b200-longctx": replace(_d(16, 16, 2, 2048, 5504), block_size=32768, init_std=0.02),
}


def get_preset(name: str) -> ModelConfig:
    key = name if name in PRESETS else name.upper()
    if key not in PRESETS:
        for k in PRESETS:
            if k.lower() == name.lower():
                key = k
                break
    if key not in PRESETS:
        raise KeyError(f"unknown model preset {name!r}; known: {sorted(PRESETS)}")
    return PRESETS[key]
