"""Dense SwiGLU MLP and top-k MoE (reference: tinytron/model/modules/mlp.py:16-297).

MLP: down(silu(gate(x)) * up(x)), no bias.  On CUDA gate|up is one tcgen05 GEMM with
the SwiGLU epilogue and the backward's SwiGLU derivative runs in the down-proj
dgrad epilogue.

MoE: router linear -> top-k over logits -> softmax over the k selected logits ->
experts (SwiGLU) -> weighted sum over k.  Expert weights keep the reference's
shapes and names ([E_local, I, H] gate/up, [E_local, H, I] down) and the
``nn.Linear`` convention y = x W^T (the reference's padded-bmm path; its
grouped_mm path multiplies untransposed and only works for I == H).  With EP > 1
tokens are dispatched to the owning rank with a variable all-to-all and combined
back (training); cached inference computes local experts only and all-reduces.
"""
from __future__ import annotations

import os
import time

import torch
import torch.distributed as dist
import torch.nn as nn

from tinytron_b200 import ops
from tinytron_b200.parallel import parallel_state
from tinytron_b200.parallel.expert_parallel import ep_all_to_all, ep_all_to_all_no_grad

from .norm import default_device


class MLP(nn.Module):
    def __init__(self, config, layer_idx: int, use_moe: bool = False, device=None):
        super().__init__()
        device = device if device is not None else default_device()
        self.config = config
        self.layer_idx = layer_idx
        self.hidden_size = config.hidden_size
        self.intermediate_size = config.moe_intermediate_size if use_moe else config.intermediate_size
        self.use_moe = use_moe
        H, I = self.hidden_size, self.intermediate_size
        self.gate_proj = nn.Linear(H, I, bias=False, device=device)
        self.up_proj = nn.Linear(H, I, bias=False, device=device)
        self.down_proj = nn.Linear(I, H, bias=False, device=device)
        self.act_fn = nn.SiLU()
        dev = self.gate_proj.weight.device
        for lin in (self.gate_proj, self.up_proj, self.down_proj):  # reference mlp.py:33-42 seeding
            with torch.random.fork_rng(devices=[dev] if dev.type == "cuda" else []):
                torch.manual_seed(config.seed + layer_idx)
                nn.init.normal_(lin.weight, mean=0.0, std=config.init_std)

    def forward(self, x: torch.Tensor, use_cache: bool = False) -> torch.Tensor:
        return ops.swiglu_mlp(x, self.gate_proj.weight, self.up_proj.weight, self.down_proj.weight)


def _ep_context():
    g = parallel_state.get_sp_group_or_none()
    if g is None or not dist.is_initialized():
        return None, 1, 0
    return g, parallel_state.get_ep_world_size(), parallel_state.get_ep_rank()


class MoE(nn.Module):
    def __init__(self, config, layer_idx: int, top_k: int | None = None, device=None):
        super().__init__()
        device = device if device is not None else default_device()
        self.config = config
        self.layer_idx = layer_idx
        self.num_experts = config.num_experts
        self.top_k = top_k if top_k is not None else config.num_experts_per_tok
        assert self.top_k <= self.num_experts, "top_k must be <= num_experts"
        self.hidden_size = config.hidden_size
        self.intermediate_size = config.moe_intermediate_size
        self.router = nn.Linear(self.hidden_size, self.num_experts, bias=False, device=device)
        _, self.ep_size, ep_rank = _ep_context()
        assert self.num_experts % self.ep_size == 0
        if torch.device(device).type == "cuda" and self.num_experts % 8:
            # router logits rows must be 16-byte aligned for the TMA-fed GEMM epilogue
            raise ValueError(f"num_experts ({self.num_experts}) must be a multiple of 8 on CUDA")
        self.num_local_experts = self.num_experts // self.ep_size
        E, I, H = self.num_local_experts, self.intermediate_size, self.hidden_size
        self.experts_gate_weights = nn.Parameter(torch.empty(E, I, H, device=device))
        self.experts_up_weights = nn.Parameter(torch.empty(E, I, H, device=device))
        self.experts_down_weights = nn.Parameter(torch.empty(E, H, I, device=device))
        self.experts_act_fn = nn.SiLU()
        self._init_expert_weights(config.seed, layer_idx, ep_rank)

    def _init_expert_weights(self, base_seed: int, layer_idx: int, ep_rank: int):
        # Reference mlp.py:100-122: expert e of layer l is drawn with seed base+l+e_global.
        dev = self.experts_gate_weights.device
        with torch.random.fork_rng(devices=[dev] if dev.type == "cuda" else []):
            for le in range(self.num_local_experts):
                torch.manual_seed(base_seed + layer_idx + ep_rank * self.num_local_experts + le)
                nn.init.normal_(self.experts_gate_weights[le], mean=0.0, std=self.config.init_std)
                nn.init.normal_(self.experts_up_weights[le], mean=0.0, std=self.config.init_std)
                nn.init.normal_(self.experts_down_weights[le], mean=0.0, std=self.config.init_std)
        with torch.random.fork_rng(devices=[dev] if dev.type == "cuda" else []):
            torch.manual_seed(base_seed + layer_idx)
            nn.init.normal_(self.router.weight, mean=0.0, std=self.config.init_std)

    def _trace(self, message: str, *, sync: bool = False) -> None:
        if os.environ.get("TINYTRON_MOE_TRACE", "0") != "1":
            return
        if sync and torch.cuda.is_available():
            torch.cuda.synchronize()
        rank = dist.get_rank() if dist.is_initialized() else 0
        print(f"[moe-trace {time.strftime('%H:%M:%S')} rank={rank} layer={self.layer_idx}] {message}", flush=True)

    def _zero_expert_weight_dependency(self) -> torch.Tensor:
        return (self.experts_gate_weights.reshape(-1)[0] + self.experts_up_weights.reshape(-1)[0]
                + self.experts_down_weights.reshape(-1)[0]) * 0.0

    def route(self, x: torch.Tensor):
        """gate_logits [N, E], top-k weights [N, k] (softmax over the selected logits), ids [N, k]."""
        gate_logits = ops.linear(x, self.router.weight)
        weights, sel = ops.moe_topk_softmax(gate_logits, self.top_k)
        return gate_logits, weights, sel.long() if not x.is_cuda else sel

    def _apply_local_experts(self, rx: torch.Tensor, rexp: torch.Tensor) -> torch.Tensor:
        """rx [R, H] rows routed here with global expert ids rexp [R] -> expert outputs [R, H]."""
        if rx.shape[0] == 0:
            return rx.reshape(0, self.hidden_size) + self._zero_expert_weight_dependency().to(rx.dtype)
        if rx.is_cuda:  # grouped tcgen05 GEMMs over device-built expert segments
            local = (rexp % self.num_local_experts).to(torch.int32).view(-1, 1)
            return ops.moe_experts(rx, local, None, self.experts_gate_weights, self.experts_up_weights,
                                   self.experts_down_weights)
        local = rexp % self.num_local_experts
        order = torch.argsort(local, stable=True)
        xs = rx[order]
        counts = torch.bincount(local, minlength=self.num_local_experts).tolist()
        outs = []
        start = 0
        for e, c in enumerate(counts):
            if c == 0:
                continue
            outs.append(ops.swiglu_mlp(xs[start:start + c], self.experts_gate_weights[e],
                                       self.experts_up_weights[e], self.experts_down_weights[e]))
            start += c
        ys = torch.cat(outs, 0)
        out = torch.empty_like(ys)
        out[order] = ys
        return out

    def _forward_sep_local_reduce_inference(self, flat_x, sel, weights, ep_group, ep_rank, B, T):
        """Head-parallel (SEP) inference (reference mlp.py:193-222): every rank holds all
        tokens, computes the pairs routed to its own experts and the partial sums are
        all-reduced.  On CUDA this is device-only (grouped GEMMs over the local segments,
        graph-capturable heap all-reduce); the CPU path selects the local pairs eagerly."""
        D = self.hidden_size
        from tinytron_b200.parallel.symm import row_parallel_all_reduce, row_parallel_target

        if flat_x.is_cuda:
            # decode-sized batches: the combine publishes straight into the heap all-reduce
            y, reduced = ops.moe_experts_local_published(
                flat_x, sel, weights, self.experts_gate_weights, self.experts_up_weights, self.experts_down_weights,
                ep_rank * self.num_local_experts, row_parallel_target(ep_group))
            return (y if reduced else row_parallel_all_reduce(y, ep_group)).reshape(B, T, D)
        tgt = sel // self.num_local_experts
        mask = tgt == ep_rank
        partial = flat_x.new_zeros((flat_x.size(0), D))
        idx = torch.nonzero(mask.reshape(-1), as_tuple=False).squeeze(-1)
        if idx.numel() > 0:
            tok = idx // self.top_k
            out = self._apply_local_experts(flat_x[tok], sel.reshape(-1)[idx])
            partial = partial.index_put((tok,), (out.float() * weights.reshape(-1)[idx, None]).to(partial.dtype),
                                        accumulate=True)
        return row_parallel_all_reduce(partial, ep_group).reshape(B, T, D)

    def forward(self, x: torch.Tensor, use_cache: bool = False):
        B, T, D = x.shape
        ep_group, ep, ep_rank = _ep_context()
        gate_logits, weights, sel = self.route(x.reshape(B * T, D))
        self.last_selected = sel  # the load-balancing statistics reuse the router's top-k
        flat_x = x.reshape(B * T, D)
        if use_cache and ep > 1:
            return self._forward_sep_local_reduce_inference(flat_x, sel, weights, ep_group, ep_rank, B, T), \
                gate_logits.view(B, T, -1)
        if ep == 1 and x.is_cuda:  # routing, layout, grouped GEMMs and the weighted sum all on device
            y = ops.moe_experts(flat_x, sel, weights, self.experts_gate_weights, self.experts_up_weights,
                                self.experts_down_weights)
            return y.view(B, T, D), gate_logits.view(B, T, -1)
        if ep > 1 and x.is_cuda and parallel_state.native_comm_enabled():
            # dispatch/combine by NVLink peer stores/loads around the grouped GEMMs
            from tinytron_b200.parallel.ep_comm import ep_moe

            # The expert weights are inputs of the EP autograd function, which writes their
            # gradients into the fp32 main grads itself (even for experts that received no
            # rows), so no zero-valued dependency on them is added: its backward would build
            # a full-size fp32 zero gradient per weight every micro-step that nothing reads.
            y = ep_moe(flat_x, sel, weights, self.experts_gate_weights, self.experts_up_weights,
                       self.experts_down_weights, ep_group)
            return y.view(B, T, D), gate_logits.view(B, T, -1)
        rep_x = flat_x.repeat_interleave(self.top_k, dim=0)
        exp_ids = sel.reshape(-1).long()
        if ep > 1:
            tgt = exp_ids // self.num_local_experts
            gorder = torch.argsort(tgt, stable=True)
            send = torch.bincount(tgt, minlength=ep)
            recv = torch.empty_like(send)
            dist.all_to_all_single(recv, send, group=ep_group)
            send_l, recv_l = torch.stack([send, recv]).cpu().tolist()
            rx = ep_all_to_all(rep_x[gorder], send_l, recv_l, ep_group)
            rexp = ep_all_to_all_no_grad(exp_ids[gorder], send_l, recv_l, ep_group)
            out = self._apply_local_experts(rx, rexp)
            back = ep_all_to_all(out, recv_l, send_l, ep_group)
            unperm = torch.empty_like(back)
            unperm[gorder] = back
        else:
            unperm = self._apply_local_experts(rep_x, exp_ids)
        y = (unperm.float() * weights.reshape(-1, 1)).view(B * T, self.top_k, D).sum(1)
        if self.training:
            y = y + self._zero_expert_weight_dependency()
        return y.to(x.dtype if not x.is_cuda else torch.bfloat16).view(B, T, D), gate_logits.view(B, T, -1)
