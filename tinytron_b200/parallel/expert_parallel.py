"""Expert-parallel all-to-all (reference: tinytron/distributed/expert_parallel/comm.py:22-164).

Variable-split autograd all-to-all over the EP (= SEP) group: forward sends rows by
``input_splits`` and receives ``output_splits``; backward runs the reverse exchange.
Zero-row splits are legal (NCCL handles empty messages), so the reference's
pad-to-one-row and all_gather fallbacks are not needed.  ``TINYTRON_EP_TRACE=1``
prints per-rank trace lines like the reference.
"""
from __future__ import annotations

import os
import time

import torch
import torch.distributed as dist


def _trace(message: str, tensor: torch.Tensor | None = None, *, sync: bool = False) -> None:
    if os.environ.get("TINYTRON_EP_TRACE", "0") != "1":
        return
    if sync and tensor is not None and tensor.is_cuda:
        torch.cuda.synchronize(tensor.device)
    rank = dist.get_rank() if dist.is_initialized() else 0
    print(f"[ep-trace {time.strftime('%H:%M:%S')} rank={rank}] {message}", flush=True)


def _a2a(x: torch.Tensor, in_splits, out_splits, group) -> torch.Tensor:
    x = x.contiguous()
    out = x.new_empty((int(sum(out_splits)),) + tuple(x.shape[1:]))
    dist.all_to_all_single(out, x, output_split_sizes=[int(s) for s in out_splits],
                           input_split_sizes=[int(s) for s in in_splits], group=group)
    return out


class EPAllToAll(torch.autograd.Function):
    @staticmethod
    def forward(ctx, hidden_states, input_splits, output_splits, ep_group):
        ctx.splits = (list(input_splits), list(output_splits))
        ctx.group = ep_group
        _trace(f"forward input={list(map(int, input_splits))} output={list(map(int, output_splits))}", hidden_states)
        return _a2a(hidden_states, input_splits, output_splits, ep_group)

    @staticmethod
    def backward(ctx, grad_output):
        ins, outs = ctx.splits
        _trace(f"backward input={outs} output={ins}", grad_output)
        return _a2a(grad_output, outs, ins, ctx.group), None, None, None


def ep_all_to_all(hidden_states, input_splits, output_splits, ep_group):
    return EPAllToAll.apply(hidden_states, input_splits, output_splits, ep_group)


def ep_all_to_all_no_grad(tensor, input_splits, output_splits, ep_group):
    with torch.no_grad():
        return _a2a(tensor, input_splits, output_splits, ep_group)
