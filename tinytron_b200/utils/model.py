"""Parameter-count helpers (reference: tinytron/utils/model.py:5-178)."""
from __future__ import annotations


def get_model_params(model_config):
    c = model_config
    if c.use_moe:
        k = c.num_experts_per_tok if isinstance(c.num_experts_per_tok, int) else max(c.num_experts_per_tok)
        return get_moe_model_params(c.num_layer, c.hidden_size, c.intermediate_size, c.vocab_size, c.num_experts, k,
                                    c.moe_intermediate_size)
    return get_dense_model_params(c.num_layer, c.hidden_size, c.intermediate_size, c.vocab_size)


def get_dense_model_params(num_layer, hidden_size, intermediate_size, vocab_size):
    """Approximate counts in billions: tied embedding + L * (4H^2 + 3HI)."""
    H, L, I, V = hidden_size, num_layer, intermediate_size, vocab_size
    total = V * H + L * (4 * H * H + 3 * H * I)
    return {"total_params_B": total / 1e9, "dense_params_B": total / 1e9}


def get_moe_model_params(num_layer, hidden_size, intermediate_size, vocab_size, num_expert, top_k,
                         moe_intermediate_size):
    """Approximate counts in billions (same accounting as the reference: dense part uses
    4H^2 + 2HI per layer, experts 3*H*I_moe each)."""
    H, L, I, E, k, Im, V = hidden_size, num_layer, intermediate_size, num_expert, top_k, moe_intermediate_size, vocab_size
    embed = V * H
    dense = L * (4 * H * H + 2 * H * I)
    router = L * H * E
    expert = 3 * H * Im
    moe_all, moe_active = L * E * expert, L * k * expert
    return {
        "total_params_B": (embed + dense + router + moe_all) / 1e9,
        "active_params_B": (embed + dense + router + moe_active) / 1e9,
        "dense_params_B": (embed + dense + router) / 1e9,
        "moe_total_B": moe_all / 1e9,
        "moe_active_B": moe_active / 1e9,
    }


def get_compiled_to_uncompiled_mapping(raw_model, compiled_keys):
    """Map checkpoint keys that may carry torch.compile's ``_orig_mod.`` prefix to the
    uncompiled model's tensors; warns about keys that match nothing."""
    sd = raw_model.state_dict()
    prefix = "_orig_mod."
    mapping = {}
    for key in compiled_keys:
        plain = key[len(prefix):] if key.startswith(prefix) else key
        if plain in sd:
            mapping[key] = sd[plain]
        else:
            print(f"Warning: Could not find a match for checkpoint key '{key}' in the model.")
    mapped = {k[len(prefix):] if k.startswith(prefix) else k for k in mapping}
    missing = set(sd) - mapped
    if missing:
        print("Warning: The following model parameters were not found in the checkpoint:")
        for k in sorted(missing)[:5]:
            print(f"  - {k}")
    return mapping
