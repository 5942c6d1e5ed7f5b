"""GQA/MHA attention with HF half-split RoPE (reference: tinytron/model/modules/attn.py:104-439).

Modes (same as the reference):
  * local training (sp == 1): fused QKV projection -> RoPE + flash attention on the
    packed buffer -> c_proj.  K/V heads are never expanded.
  * SEP training (sp > 1, Ulysses): the QKV output is transposed heads<->sequence with
    an all-to-all that routes each kv head only to the ranks that read it, attention
    runs over the full sequence for the local heads, and the inverse all-to-all
    returns the local sequence chunk for all heads before c_proj.
  * KV-cache inference (``use_cache``): prefill/decode with a paged or concatenated
    cache; with sp > 1 each SEP rank owns Hq/sp heads ("head-parallel decode"),
    multiplies by its c_proj column slice and all-reduces (row-parallel).
    ``inference_shard_qkv`` sizes q/k/v to the local heads.

Positions are global: rank r of an SP group holding chunk r uses r*T_local + t
(reference attn.py:393); decode uses position_offset.
"""
from __future__ import annotations

import math

import torch
import torch.distributed as dist
import torch.nn as nn
import torch.nn.functional as F

from tinytron_b200 import ops
from tinytron_b200.ops.rope import rope_reference
from tinytron_b200.parallel import parallel_state
from tinytron_b200.parallel.ulysses import gather_heads_from_ranks, route_heads_to_ranks

from .norm import default_device


def rope_impl(q, k, position_ids, rope_theta: float = 10000.0):
    """Reference-compatible functional RoPE on [B, H, T, D] tensors."""
    return rope_reference(q, k, position_ids, rope_theta)


def gqa_impl(k, v, num_key_value_heads: int, num_attention_heads: int):
    """Expand [B, Hkv, T, D] to [B, Hq, T, D] (API parity; the kernels never need it)."""
    if num_key_value_heads == num_attention_heads:
        return k, v
    if num_attention_heads % num_key_value_heads:
        raise ValueError("num_attention_heads must be divisible by num_key_value_heads")
    r = num_attention_heads // num_key_value_heads
    return k.repeat_interleave(r, dim=1), v.repeat_interleave(r, dim=1)


def build_cache_causal_mask(query_len: int, key_len: int, past_len: int, device) -> torch.Tensor:
    q = past_len + torch.arange(query_len, device=device).unsqueeze(-1)
    return torch.arange(key_len, device=device).unsqueeze(0) <= q


def _is_paged_kv_cache(past_kv) -> bool:
    return hasattr(past_kv, "append") and hasattr(past_kv, "get_kv") and hasattr(past_kv, "current_length")


def sp_context():
    g = parallel_state.get_sp_group_or_none()
    if g is None or not dist.is_initialized():
        return None, 1, 0
    return g, parallel_state.get_sp_world_size(), parallel_state.get_sp_rank()


class Attention(nn.Module):
    def __init__(self, config, layer_idx: int, device=None):
        super().__init__()
        assert config.hidden_size % config.num_attention_heads == 0
        device = device if device is not None else default_device()
        self.config = config
        self.layer_idx = layer_idx
        self.num_attention_heads = config.num_attention_heads
        self.num_key_value_heads = config.num_key_value_heads
        self.head_dim = config.hidden_size // config.num_attention_heads
        self.n_embd = config.hidden_size
        self.dropout = config.dropout
        self.rope_theta = float(getattr(config, "rope_theta", 10000.0))
        self.inference_shard_qkv = bool(config.inference_shard_qkv)
        self.q_proj_heads = self.num_attention_heads
        self.kv_proj_heads = self.num_key_value_heads
        if self.inference_shard_qkv:
            sp = parallel_state.get_sp_world_size()
            if sp > 1:
                if self.num_attention_heads % sp or self.num_key_value_heads % sp:
                    raise ValueError(
                        f"num_attention_heads ({self.num_attention_heads}) and num_key_value_heads "
                        f"({self.num_key_value_heads}) must be divisible by sp_size ({sp}) for inference_shard_qkv.")
                self.q_proj_heads = self.num_attention_heads // sp
                self.kv_proj_heads = self.num_key_value_heads // sp
        D = config.hidden_size
        self.q_proj = nn.Linear(D, self.q_proj_heads * self.head_dim, bias=False, device=device)
        self.k_proj = nn.Linear(D, self.kv_proj_heads * self.head_dim, bias=False, device=device)
        self.v_proj = nn.Linear(D, self.kv_proj_heads * self.head_dim, bias=False, device=device)
        self.c_proj = nn.Linear(D, D, bias=False, device=device)
        self._init_weights(config.seed, layer_idx)

    def _init_weights(self, base_seed: int, layer_idx: int):
        # Same seeding scheme as the reference (attn.py:148-160): every projection is
        # drawn after reseeding with seed + layer_idx.
        dev = self.q_proj.weight.device
        for lin in (self.q_proj, self.k_proj, self.v_proj, self.c_proj):
            with torch.random.fork_rng(devices=[dev] if dev.type == "cuda" else []):
                torch.manual_seed(base_seed + layer_idx)
                nn.init.normal_(lin.weight, mean=0.0, std=self.config.init_std)

    # ------------------------------------------------------------------ training
    def forward_train(self, h: torch.Tensor, position_offset: int = 0) -> torch.Tensor:
        """h [B, T_local, D] -> attention output [B, T_local, D] (no cache)."""
        B, T, D = h.shape
        Hq, Hkv, hd = self.num_attention_heads, self.num_key_value_heads, self.head_dim
        sp_group, sp, sp_rank = sp_context()
        qkv = ops.linear(h, self.q_proj.weight, self.k_proj.weight, self.v_proj.weight)
        qkv = qkv.reshape(B * T, (Hq + 2 * Hkv) * hd)
        if sp == 1:
            o = ops.rotary_attention(qkv, B, T, Hq, Hkv, hd, position_offset, self.rope_theta, causal=True)
            return ops.linear(o.view(B, T, Hq * hd), self.c_proj.weight)
        if Hq % sp:
            raise AssertionError(f"Attention heads ({Hq}) must be divisible by sp_size ({sp})")
        full, hq_l, hkv_l = route_heads_to_ranks(qkv, B, T, Hq, Hkv, hd, sp, sp_group)
        o = ops.rotary_attention(full, B, T * sp, hq_l, hkv_l, hd, position_offset, self.rope_theta, causal=True)
        y = gather_heads_from_ranks(o, B, T, Hq, hd, sp, sp_group)
        return ops.linear(y, self.c_proj.weight)

    # ------------------------------------------------------------------ generic / cached
    def forward(self, x: torch.Tensor, past_kv=None, use_cache: bool = False, position_offset: int = 0):
        if not use_cache and past_kv is None:
            return self.forward_train(x, position_offset), None
        return self._forward_cached(x, past_kv, use_cache, position_offset)

    def _local_heads(self, sp: int, sp_rank: int):
        """(q head range, kv head range) owned by this rank in head-parallel decode."""
        Hq, Hkv = self.num_attention_heads, self.num_key_value_heads
        if sp == 1:
            return (0, Hq), (0, Hkv)
        hq_l = Hq // sp
        G = Hq // Hkv
        q0 = sp_rank * hq_l
        return (q0, q0 + hq_l), (q0 // G, (q0 + hq_l - 1) // G + 1)

    def _forward_cached(self, x, past_kv, use_cache, position_offset):
        B, T, D = x.shape
        hd = self.head_dim
        sp_group, sp, sp_rank = sp_context()
        if sp > 1 and self.num_attention_heads % sp:
            raise AssertionError(f"Attention heads ({self.num_attention_heads}) must be divisible by sp_size ({sp})")
        (q0, q1), (k0, k1) = self._local_heads(sp, sp_rank)
        if self.inference_shard_qkv or sp == 1:
            wq, wk, wv = self.q_proj.weight, self.k_proj.weight, self.v_proj.weight
        else:
            wq = self.q_proj.weight[q0 * hd:q1 * hd]
            wk = self.k_proj.weight[k0 * hd:k1 * hd]
            wv = self.v_proj.weight[k0 * hd:k1 * hd]
        hq_l, hkv_l = q1 - q0, k1 - k0
        qkv = ops.linear(x, wq, wk, wv).reshape(B, T, hq_l + 2 * hkv_l, hd)
        q = qkv[:, :, :hq_l].transpose(1, 2)
        k = qkv[:, :, hq_l:hq_l + hkv_l].transpose(1, 2)
        v = qkv[:, :, hq_l + hkv_l:].transpose(1, 2)
        G = self.num_attention_heads // self.num_key_value_heads
        if self._fused_cache_ok(x, past_kv, position_offset, q0, k0, hq_l, hkv_l, G, sp):
            return self._forward_cached_fused(qkv, past_kv, B, T, hq_l, hkv_l, q0, q1, sp, sp_group, use_cache)
        if sp > 1 and not self.inference_shard_qkv:
            true_map = [(q0 + i) // G - k0 for i in range(hq_l)]
            ratio = hq_l // hkv_l if hq_l % hkv_l == 0 else 0
            if ratio == 0 or any(true_map[i] != i // ratio for i in range(hq_l)):
                # this rank's q heads do not map uniformly onto its kv heads: expand them
                idx = torch.tensor(true_map, device=x.device)
                k, v, hkv_l = k.index_select(1, idx), v.index_select(1, idx), hq_l
        pos = torch.arange(position_offset, position_offset + T, device=x.device).unsqueeze(0)
        q, k = rope_reference(q, k, pos, self.rope_theta)
        if _is_paged_kv_cache(past_kv):
            past_len = past_kv.append(k, v)
            k_all, v_all = past_kv.get_kv()
            new_kv = past_kv
        elif past_kv is not None:
            past_len = past_kv[0].size(2)
            k_all = torch.cat([past_kv[0], k.to(past_kv[0].dtype)], dim=2)
            v_all = torch.cat([past_kv[1], v.to(past_kv[1].dtype)], dim=2)
            new_kv = (k_all, v_all)
        else:
            past_len = 0
            k_all, v_all = k, v
            new_kv = (k_all, v_all)
        y = self._cached_attention(q, k_all, v_all, past_len, hq_l, hkv_l)  # [B, T, hq_l*hd]
        if sp > 1:
            wc = self.c_proj.weight[:, q0 * hd:q1 * hd]
            y = ops.linear(y, wc)
            dist.all_reduce(y, op=dist.ReduceOp.SUM, group=sp_group)
        else:
            y = ops.linear(y, self.c_proj.weight)
        return y, (new_kv if use_cache else None)

    # ------------------------------------------------------------------ fused CUDA cache path
    def _fused_cache_ok(self, x, past_kv, position_offset, q0, k0, hq_l, hkv_l, G, sp) -> bool:
        """Paged cache on CUDA whose q heads map uniformly onto its kv heads (no
        expansion) and whose length equals the requested position."""
        if not (x.is_cuda and _is_paged_kv_cache(past_kv) and self.head_dim in (64, 128)):
            return False
        if position_offset != past_kv.current_length or hq_l % hkv_l or hq_l // hkv_l > 8:
            return False
        if sp > 1 and not self.inference_shard_qkv:
            ratio = hq_l // hkv_l
            if any((q0 + i) // G - k0 != i // ratio for i in range(hq_l)):
                return False
        return True

    def _forward_cached_fused(self, qkv, past_kv, B, T, hq_l, hkv_l, q0, q1, sp, sp_group, use_cache):
        """RoPE + paged append in one kernel; decode (T == 1) attends straight from the
        pages (split-KV kernel); prefill attends over the new tokens with the flash
        kernel.  Graph-capturable for T == 1 (positions come from the cache's device
        length)."""
        from tinytron_b200.ops import _ext
        from tinytron_b200.ops.functional import attention_fwd_only
        from tinytron_b200.ops.rope import rope_tables

        hd = self.head_dim
        qkv2 = qkv.reshape(B * T, (hq_l + 2 * hkv_l) * hd)
        past_len = past_kv.current_length
        q = past_kv.append_rope(qkv2, B, T, hq_l, hkv_l, hd, self.rope_theta)
        if T == 1:
            y = past_kv.attend_decode(q.view(B, hq_l, hd), 1.0 / math.sqrt(hd)).view(B, 1, hq_l * hd)
        elif past_len == 0:
            cos, sin = rope_tables(hd, self.rope_theta, past_kv.max_seq_len, qkv.device)
            qkv_r = qkv2.contiguous().clone()
            _ext.load().rope_inplace(qkv_r, cos, sin, T, 0, hq_l + hkv_l, hd, False)
            o, _ = attention_fwd_only(qkv_r, qkv_r, qkv_r, 0, hq_l * hd, (hq_l + hkv_l) * hd, B, T, T, hq_l, hkv_l,
                                      hd, True, 0)
            y = o.view(B, T, hq_l * hd)
        else:
            k_all, v_all = past_kv.gather_tokens(past_len + T)  # [B, L, Hkv, D], includes the new tokens
            L = past_len + T
            o, _ = attention_fwd_only(q, k_all.reshape(B * L, hkv_l * hd).contiguous(),
                                      v_all.reshape(B * L, hkv_l * hd).contiguous(), 0, 0, 0, B, T, L, hq_l, hkv_l,
                                      hd, True, past_len)
            y = o.view(B, T, hq_l * hd)
        past_kv.advance(T)
        if sp > 1:
            from tinytron_b200.ops.weights import bf16_of
            from tinytron_b200.parallel.symm import row_parallel_all_reduce, row_parallel_target

            ar = row_parallel_target(sp_group)
            fused = None
            if ar is not None:  # c_proj's split sums published straight into the all-reduce slot
                fused = ops.linear_row_parallel(y, bf16_of(self.c_proj.weight)[:, q0 * hd:q1 * hd], ar)
            if fused is not None:
                y = fused
            else:
                y = row_parallel_all_reduce(ops.linear(y, self.c_proj.weight[:, q0 * hd:q1 * hd]), sp_group)
        else:
            y = ops.linear(y, self.c_proj.weight)
        return y, (past_kv if use_cache else None)

    def _cached_attention(self, q, k_all, v_all, past_len, hq_l, hkv_l):
        B, _, T, hd = q.shape
        L = k_all.size(2)
        if q.is_cuda and hd in (64, 128):
            qt = q.transpose(1, 2).reshape(B * T, hq_l * hd).to(torch.bfloat16).contiguous()
            kt = k_all.transpose(1, 2).reshape(B * L, hkv_l * hd).to(torch.bfloat16).contiguous()
            vt = v_all.transpose(1, 2).reshape(B * L, hkv_l * hd).to(torch.bfloat16).contiguous()
            from tinytron_b200.ops.functional import attention_fwd_only

            o, _ = attention_fwd_only(qt, kt, vt, 0, 0, 0, B, T, L, hq_l, hkv_l, hd, True, past_len)
            return o.view(B, T, hq_l * hd)
        k_e, v_e = gqa_impl(k_all, v_all, hkv_l, hq_l)
        if past_len > 0:
            mask = build_cache_causal_mask(T, L, past_len, q.device)
            o = F.scaled_dot_product_attention(q, k_e.to(q.dtype), v_e.to(q.dtype), attn_mask=mask)
        else:
            o = F.scaled_dot_product_attention(q, k_e.to(q.dtype), v_e.to(q.dtype), is_causal=True)
        return o.transpose(1, 2).reshape(B, T, hq_l * hd)
