"""GPT / MoE language model (reference: tinytron/model/gpt.py:20-163).

Module tree, parameter names and init seeding match the reference, so state dicts
interoperate (``wte``, ``blocks.{l}.{ln_1,attn,ln_2,mlp}``, ``lnf``, tied ``lm_head``).

Training forward (no cache) runs the fused path: each residual add is folded into
the following RMSNorm (fp32 residual stream, bf16 normalised output), attention
reads Q/K/V straight from the fused QKV projection, and the LM head is fused with
the cross-entropy so the full logits never materialise in fp32.  With ``targets``
the return value is ``(logits, loss + aux_loss, logging_loss)`` like the reference;
``logits`` is None unless ``return_logits=True`` (computing them costs an extra
[tokens x vocab] GEMM and buffer).
"""
from __future__ import annotations

import os

import torch
import torch.distributed as dist
import torch.nn as nn

from tinytron_b200 import ops
from tinytron_b200.utils.profile import nvtx_range
from tinytron_b200.parallel import parallel_state

from .config import ModelConfig
from .modules.attn import Attention
from .modules.loss import CrossEntropyLoss, ExpertLoadBalancingLoss
from .modules.mlp import MLP, MoE
from .modules.norm import LayerNorm, default_device

EXPERT_LOCAL_PARAM_SUFFIXES = (
    "mlp.experts_gate_weights",
    "mlp.experts_up_weights",
    "mlp.experts_down_weights",
)


class Block(nn.Module):
    def __init__(self, config: ModelConfig, layer_idx: int, use_moe: bool = True, top_k: int | None = None,
                 device=None):
        super().__init__()
        self.config = config
        self.layer_idx = layer_idx
        self.use_moe = use_moe
        self.ln_1 = LayerNorm(config, device)
        self.attn = Attention(config, layer_idx, device)
        self.ln_2 = LayerNorm(config, device)
        self.mlp = MoE(config, layer_idx, top_k, device) if use_moe else MLP(config, layer_idx, device=device)

    def forward(self, x, past_kv=None, use_cache: bool = False, position_offset: int = 0):
        a, new_kv = self.attn(self.ln_1(x), past_kv=past_kv, use_cache=use_cache, position_offset=position_offset)
        x = x + a
        out = self.mlp(self.ln_2(x), use_cache=use_cache)
        if self.use_moe:
            return x + out[0], out[1], new_kv
        return x + out, None, new_kv


class GPT(nn.Module):
    def __init__(self, config: ModelConfig, device=None):
        super().__init__()
        device = torch.device(device) if device is not None else default_device()
        self.device = device
        self.config = config
        self.use_moe = config.use_moe
        self.eps = float(getattr(config, "rms_norm_eps", 1e-6))
        self.wte = nn.Embedding(config.vocab_size, config.hidden_size, device=device)
        self.blocks = nn.ModuleList([Block(config, i, self.use_moe, device=device) for i in range(config.num_layer)])
        self.lnf = LayerNorm(config, device)
        self.lm_head = nn.Linear(config.hidden_size, config.vocab_size, bias=False, device=device)
        if config.tied_lm_head:
            self.lm_head.weight = self.wte.weight
        self.loss_fn = CrossEntropyLoss()
        # TT_LM_HEAD_CHUNK_ROWS=n: LM head + CE in chunks of n rows recomputed in the backward
        # (no [tokens, vocab] logits buffer); 0 keeps the single fused pass (fastest).
        self.lm_head_chunk_rows = int(os.environ.get("TT_LM_HEAD_CHUNK_ROWS", "0") or 0)
        self.expert_loss_fn = (
            ExpertLoadBalancingLoss(config.num_experts, config.num_experts_per_tok, alpha=config.moe_balance_loss_weight)
            if config.use_moe and config.moe_balance_loss_weight > 0.0 else None)
        self._init_weights(config.seed)

    def _init_weights(self, base_seed: int):
        dev = self.wte.weight.device
        fork = [dev] if dev.type == "cuda" else []
        with torch.random.fork_rng(devices=fork):
            torch.manual_seed(base_seed)
            nn.init.normal_(self.wte.weight, mean=0.0, std=self.config.init_std)
        if not self.config.tied_lm_head:
            with torch.random.fork_rng(devices=fork):
                torch.manual_seed(base_seed)
                nn.init.normal_(self.lm_head.weight, mean=0.0, std=self.config.init_std)

    # ------------------------------------------------------------------ forward
    def forward(self, idx, targets=None, past_key_values=None, use_cache: bool = False, position_offset: int = 0,
                return_logits: bool = False):
        B, T = idx.size()
        assert T <= self.config.block_size, f"Cannot forward sequence of length {T}, block size is only {self.config.block_size}"
        if use_cache or past_key_values is not None:
            return self._forward_cached(idx, past_key_values, use_cache, position_offset)
        aux_stats = [] if targets is not None and self.expert_loss_fn is not None else None
        h, _ = self._trunk(idx, targets, position_offset, aux_stats=aux_stats)
        if targets is None:
            if torch.is_grad_enabled():  # differentiable logits (e.g. RL policy log-probs)
                return ops.linear(h, self.lm_head.weight)
            return ops.lm_logits(h, self.lm_head.weight)
        valid = targets != self.loss_fn.ignore_index
        loss_sum = ops.lm_head_ce_sum(h, self.lm_head.weight, targets, self.loss_fn.ignore_index,
                                      chunk_rows=self.lm_head_chunk_rows)
        loss, logging_loss, total_aux = self._reduce_step_stats(loss_sum, valid.sum(), aux_stats)
        logits = None
        if return_logits:
            with torch.no_grad():
                logits = ops.lm_logits(h.detach(), self.lm_head.weight)
        return logits, loss + total_aux, logging_loss

    def _reduce_step_stats(self, loss_sum, valid_count, aux_stats):
        """Every cross-rank statistic of the forward in ONE packed all-reduce over DP x SP
        (the reference issues one per quantity and two per MoE layer): the MoE selection
        counts of every layer, and one slot per rank for the valid-token count, the local
        loss sum and the routed-token count, from which the SP/EP-group sums follow.
        Also leaves (SP-group valid tokens, DP x SP valid tokens) in ``last_token_counts``
        for the trainer's loss weighting."""
        from tinytron_b200.parallel.scalars import all_reduce_scalars

        group = parallel_state._DP_SP_GROUP
        world = parallel_state.get_dp_sp_world_size()
        me = parallel_state.get_dp_sp_rank()
        # the SEP group is a contiguous block of ranks (parallel_state's layout): a slice, so
        # no index tensor is built (a host-to-device copy would synchronise every micro-step)
        sp_ranks = parallel_state.get_sep_ranks() if group is not None else [me]
        sp_idx = slice(sp_ranks[0], sp_ranks[-1] + 1)
        E = self.config.num_experts if aux_stats else 0
        n_layers = len(aux_stats) if aux_stats else 0
        with torch.no_grad():
            vec = torch.zeros(n_layers * E + 3 * world, dtype=torch.float32, device=loss_sum.device)
            base = n_layers * E
            vec[base + me] = valid_count.float()
            vec[base + world + me] = loss_sum.detach().float()
            for li, (_, f_sum, n_local) in enumerate(aux_stats or []):
                vec[li * E:(li + 1) * E] = f_sum
                if li == 0:
                    vec[base + 2 * world + me] = n_local
            red = all_reduce_scalars(vec, group)
            counts, sums, routed = red[base:base + world], red[base + world:base + 2 * world], red[base + 2 * world:]
            sp_count = counts[sp_idx].sum().clamp(min=1.0)
            logging_loss = sums[sp_idx].sum() / sp_count
            self.last_token_counts = (counts[sp_idx].sum(), counts.sum())
        loss = loss_sum / sp_count
        total_aux = 0.0
        if aux_stats:
            tokens_ep, tokens_all = routed[sp_idx].sum(), routed.sum()
            for li, (p_sum, _, _) in enumerate(aux_stats):
                total_aux = total_aux + self.expert_loss_fn.from_global_stats(p_sum, red[li * E:(li + 1) * E],
                                                                              tokens_ep, tokens_all)
        return loss, logging_loss, total_aux

    def token_log_probs(self, idx, targets, position_offset: int = 0):
        """log p(targets[b, t] | idx[b, :t+1]) as fp32 ``[B, T]``, differentiable, without
        materialising logits beyond the fused LM-head + cross-entropy kernel's bf16 buffer
        (which its backward reuses in place).  Targets equal to the ignore index (-100)
        get log-prob 0 and no gradient.  Used by the RL trainers for the actor's log-probs."""
        h, _ = self._trunk(idx, None, position_offset)
        return ops.lm_head_token_logprobs(h, self.lm_head.weight, targets, self.loss_fn.ignore_index).view(
            targets.shape)

    def _trunk(self, idx, targets, position_offset: int = 0, aux_stats: list | None = None):
        """Embedding -> blocks -> final norm; returns (normalised hidden states, MoE aux loss).
        With ``aux_stats`` (a list) the MoE layers append their local load-balancing
        statistics there instead of reducing them one layer at a time (aux loss 0 then)."""
        x = ops.embedding(idx, self.wte.weight)
        pending = None
        total_aux = 0.0
        valid = (targets != self.loss_fn.ignore_index) if targets is not None else None
        for li, blk in enumerate(self.blocks):
            with nvtx_range(f"layer{li}.attn"):
                x, h = ops.add_rmsnorm(x, pending, blk.ln_1.weight, self.eps)
                a = blk.attn.forward_train(h, position_offset)
            with nvtx_range(f"layer{li}.mlp"):
                x, h = ops.add_rmsnorm(x, a, blk.ln_2.weight, self.eps)
                if self.use_moe:
                    pending, gate_logits = blk.mlp(h)
                    if aux_stats is not None:
                        aux_stats.append(self.expert_loss_fn.local_stats(
                            gate_logits, valid_mask=valid, selected_experts=getattr(blk.mlp, "last_selected", None)))
                    elif self.expert_loss_fn is not None and targets is not None:
                        total_aux = total_aux + self.expert_loss_fn(gate_logits, valid_mask=valid)
                else:
                    pending = blk.mlp(h)
        x, h = ops.add_rmsnorm(x, pending, self.lnf.weight, self.eps)
        return h, total_aux

    def _forward_cached(self, idx, past_key_values, use_cache, position_offset, last_only: bool = False):
        x = ops.embedding(idx, self.wte.weight)
        paged = past_key_values if hasattr(past_key_values, "get_layer_cache") else None
        new_past = paged if paged is not None else ([] if use_cache else None)
        if x.is_cuda:  # residual adds fused into the following RMSNorm, as in training
            pending = None
            for i, blk in enumerate(self.blocks):
                layer_past = paged.get_layer_cache(i) if paged is not None else (
                    past_key_values[i] if past_key_values is not None else None)
                x, h = ops.add_rmsnorm(x, pending, blk.ln_1.weight, self.eps)
                a, new_kv = blk.attn(h, past_kv=layer_past, use_cache=use_cache, position_offset=position_offset)
                x, h = ops.add_rmsnorm(x, a, blk.ln_2.weight, self.eps)
                out = blk.mlp(h, use_cache=use_cache)
                pending = out[0] if self.use_moe else out
                if use_cache and paged is None:
                    new_past.append(new_kv)
            if last_only:
                x, pending = x[:, -1:].contiguous(), pending[:, -1:].contiguous()
            _, h = ops.add_rmsnorm(x, pending, self.lnf.weight, self.eps)
            logits = ops.lm_logits(h, self.lm_head.weight)
            return (logits, new_past) if use_cache else logits
        for i, blk in enumerate(self.blocks):
            if paged is not None:
                layer_past = paged.get_layer_cache(i)
            else:
                layer_past = past_key_values[i] if past_key_values is not None else None
            x, _, new_kv = blk(x, past_kv=layer_past, use_cache=use_cache, position_offset=position_offset)
            if use_cache and paged is None:
                new_past.append(new_kv)
        if last_only:
            x = x[:, -1:]
        logits = self.lm_head(self.lnf(x)) if not x.is_cuda else ops.lm_logits(self.lnf(x), self.lm_head.weight)
        if use_cache:
            return logits, new_past
        return logits

    # ------------------------------------------------------------------ accounting
    def get_flops_per_fwd_bwd(self, batch_size, seq_len):
        """Reference FLOP formula (gpt.py:117-141): MHA-sized QKV, full (non-causal)
        attention, no LM head; used for reference-comparable MFU."""
        sp = parallel_state.get_sp_world_size()
        ep = parallel_state.get_ep_world_size()
        c = self.config
        D = c.hidden_size
        qkv_out = 8 * batch_size * seq_len * D * D
        attn_mm = 4 * batch_size * seq_len * seq_len * D
        I = c.moe_intermediate_size if self.use_moe else c.intermediate_size
        ffn = 2 * batch_size * seq_len * D * I * 3 + batch_size * seq_len * I
        gate = 2 * batch_size * seq_len * D * c.num_experts
        if self.use_moe:
            per_layer = (qkv_out + attn_mm + gate) / sp + (c.num_experts_per_tok * ffn) / ep
        else:
            per_layer = (qkv_out + attn_mm + ffn) / sp
        return 3 * c.num_layer * per_layer

    def get_flops_per_fwd_bwd_exact(self, batch_size, seq_len_local, sp: int = 1):
        """Executed FLOPs per rank per micro-step (GQA-sized QKV, causal attention, LM head)."""
        from tinytron_b200.utils.flops import training_flops_per_microstep

        return training_flops_per_microstep(self.config, batch_size, seq_len_local, sp)

    @torch.no_grad()
    def clip_grad_norm(self, max_norm: float, norm_type: float = 2):
        """Global grad-norm clip; expert grads' norm^2 is summed over the EP group
        (reference gpt.py:143-163).  Uses ``main_grad`` when the model has flat grads."""
        dev = next(self.parameters()).device
        normal_sq = torch.zeros((), device=dev)
        expert_sq = torch.zeros((), device=dev)
        grads = []
        seen = set()
        for name, p in self.named_parameters():
            if id(p) in seen:
                continue
            seen.add(id(p))
            g = p.__dict__.get("main_grad")
            if g is None:
                g = p.grad
            if g is None:
                continue
            grads.append(g)
            sq = torch.linalg.vector_norm(g, norm_type).float() ** norm_type
            if name.endswith(EXPERT_LOCAL_PARAM_SUFFIXES):
                expert_sq += sq
            else:
                normal_sq += sq
        g_ep = parallel_state.get_sp_group_or_none()
        if g_ep is not None and dist.get_world_size(g_ep) > 1:
            dist.all_reduce(expert_sq, op=dist.ReduceOp.SUM, group=g_ep)
        total = (normal_sq + expert_sq) ** (1.0 / norm_type)
        coef = torch.clamp(max_norm / (total + 1e-6), max=1.0)
        for g in grads:
            g.mul_(coef)
        return total
