"""Losses (reference: tinytron/model/modules/loss.py:9-86).

``CrossEntropyLoss``: token-mean CE whose denominator is the valid-token count
summed over the SP group (so SP shards of one sequence share one mean); also
returns a no-grad logging loss = global loss sum / global count.
``ExpertLoadBalancingLoss``: Switch-style alpha * E * sum_i f_i * P_i with f_i from
top-k selections summed over DP x SP and P_i normalised by EP-group tokens.

Both take the collectives' scalars as one packed all-reduce where possible.
"""
from __future__ import annotations

import torch
import torch.distributed as dist
import torch.nn as nn
import torch.nn.functional as F

from tinytron_b200.parallel import parallel_state


def _sp_group():
    return parallel_state.get_sp_group_or_none()


def _all_reduce(t: torch.Tensor, group) -> torch.Tensor:
    if group is not None and dist.is_initialized() and dist.get_world_size(group) > 1:
        dist.all_reduce(t, op=dist.ReduceOp.SUM, group=group)
    return t


class CrossEntropyLoss(nn.Module):
    def __init__(self, ignore_index: int = -100):
        super().__init__()
        self.ignore_index = ignore_index

    def reduce(self, local_loss_sum: torch.Tensor, local_valid_count: torch.Tensor):
        """(loss, logging_loss) from a local loss sum (with grad) and local valid count."""
        g = _sp_group()
        with torch.no_grad():
            stats = torch.stack([local_valid_count.detach().float(), local_loss_sum.detach().float()])
            _all_reduce(stats, g)
            global_count = stats[0].clamp(min=1.0)
            logging_loss = stats[1] / global_count
        loss = local_loss_sum / global_count
        return loss, logging_loss

    def forward(self, logits: torch.Tensor, targets: torch.Tensor):
        logits = logits.view(-1, logits.size(-1))
        targets = targets.view(-1)
        per = F.cross_entropy(logits, targets, ignore_index=self.ignore_index, reduction="none")
        valid = (targets != self.ignore_index).float()
        return self.reduce((per * valid).sum(), valid.sum())


class ExpertLoadBalancingLoss(nn.Module):
    def __init__(self, num_experts: int, top_k: int, alpha: float = 0.01):
        super().__init__()
        self.num_experts = num_experts
        self.top_k = top_k
        self.alpha = alpha

    def local_stats(self, gate_logits: torch.Tensor, valid_mask: torch.Tensor | None = None,
                    selected_experts: torch.Tensor | None = None):
        """This rank's part of the loss before any collective: (sum over valid tokens of
        the router softmax [E] (with grad), top-k selection counts [E] (no grad), number
        of valid tokens (0-dim, no grad)).  ``from_global_stats`` finishes the loss once the
        counts have been reduced; ``GPT.forward`` reduces every layer's counts together."""
        E = self.num_experts
        flat = gate_logits.reshape(-1, E)
        if valid_mask is not None:
            keep = valid_mask.reshape(-1).to(torch.float32)
            p_sum = (F.softmax(flat.float(), dim=-1) * keep[:, None]).sum(0)
            if selected_experts is None:
                selected_experts = torch.topk(flat, self.top_k, dim=-1).indices
            sel = selected_experts.reshape(-1, self.top_k).long()
            # selections of valid tokens: masked ones go to an extra bin (an integer count,
            # deterministic, no sort; index_add_ runs a sort-based kernel in deterministic mode)
            ids = torch.where(valid_mask.reshape(-1, 1).bool(), sel, torch.full_like(sel, E))
            f_sum = torch.bincount(ids.reshape(-1), minlength=E + 1)[:E].float()
            n_local = keep.sum()
        else:
            p_sum = F.softmax(flat.float(), dim=-1).sum(0)
            if selected_experts is None:
                selected_experts = torch.topk(flat, self.top_k, dim=-1).indices
            f_sum = torch.bincount(selected_experts.reshape(-1).long(), minlength=E).float()
            n_local = torch.tensor(float(flat.size(0)), device=flat.device)
        return p_sum, f_sum.detach(), n_local.detach()

    def from_global_stats(self, p_sum: torch.Tensor, f_global: torch.Tensor, tokens_ep: torch.Tensor,
                          tokens_global: torch.Tensor) -> torch.Tensor:
        """alpha * E * sum_i f_i * P_i with f_i = global selection share (DP x SP) and
        P_i = mean router probability over the EP group's tokens."""
        P_i = p_sum / tokens_ep.clamp(min=1.0)
        f_i = f_global / (tokens_global.clamp(min=1.0) * self.top_k)
        return self.alpha * self.num_experts * torch.sum(f_i * P_i)

    def forward(self, gate_logits: torch.Tensor, valid_mask: torch.Tensor | None = None,
                selected_experts: torch.Tensor | None = None) -> torch.Tensor:
        E = self.num_experts
        flat = gate_logits.reshape(-1, E)
        if valid_mask is not None:
            keep = valid_mask.reshape(-1).bool()
            flat = flat[keep]
            if selected_experts is not None:
                selected_experts = selected_experts.reshape(-1, self.top_k)[keep]
        n_local = flat.size(0)
        if n_local == 0:
            p_sum = flat.new_zeros(E, dtype=torch.float32)
            f_sum = flat.new_zeros(E, dtype=torch.float32)
        else:
            p_sum = F.softmax(flat.float(), dim=-1).sum(0)
            if selected_experts is None:
                selected_experts = torch.topk(flat, self.top_k, dim=-1).indices
            f_sum = torch.bincount(selected_experts.reshape(-1), minlength=E).float()
        with torch.no_grad():
            ep = parallel_state.get_sp_group_or_none()
            world = parallel_state._DP_SP_GROUP
            tok = torch.tensor([float(n_local)], device=flat.device)
            tokens_ep = _all_reduce(tok.clone(), ep).clamp(min=1.0)
            packed = torch.cat([f_sum.detach(), tok])
            _all_reduce(packed, world)
            global_f = packed[:E]
            global_tokens = packed[E].clamp(min=1.0)
        P_i = p_sum / tokens_ep
        f_i = global_f / (global_tokens * self.top_k)
        return self.alpha * E * torch.sum(f_i * P_i)
