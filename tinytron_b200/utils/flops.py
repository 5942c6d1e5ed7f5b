"""Executed-FLOP accounting for MFU: GQA-sized QKV, causal attention (half of the
full T^2 score matrix), LM head included, backward = 2x forward."""
from __future__ import annotations


def training_flops_per_microstep(config, batch_size: int, seq_len_local: int, sp: int = 1) -> float:
    c = config
    D = c.hidden_size
    hd = D // c.num_attention_heads
    tok = batch_size * seq_len_local
    qkv = 2 * tok * D * (c.num_attention_heads + 2 * c.num_key_value_heads) * hd
    proj = 2 * tok * D * D
    attn = 2 * tok * (seq_len_local * sp) * D  # QK^T + PV over the causal half
    if c.use_moe:
        ffn = c.num_experts_per_tok * 6 * tok * D * c.moe_intermediate_size + 2 * tok * D * c.num_experts
    else:
        ffn = 6 * tok * D * c.intermediate_size
    head = 2 * tok * D * c.vocab_size
    return 3.0 * (c.num_layer * (qkv + proj + attn + ffn) + head)
