"""Flat parameter / gradient / bf16-shadow buffers.

All trainable parameters of a model are re-pointed into one contiguous fp32
master buffer (``p.data`` becomes a view, so optimizers and state dicts keep
working), with a matching fp32 gradient buffer (``p.main_grad``) that the GEMM
epilogues accumulate into, and a bf16 shadow buffer the tensor-core kernels read.

Layout: non-expert parameters first, expert-local parameters last, each block
aligned to ``align`` elements (256 bytes), so
  * the SP gradient all-reduce (non-expert only) covers one contiguous prefix;
  * DP reduce-scatter / all-gather shard the whole buffer in equal contiguous chunks;
  * projections that share an input (q|k|v, gate|up) are adjacent, so their fused
    GEMMs read one [sum(out), in] weight view and write one gradient view.
"""
from __future__ import annotations

import torch

from tinytron_b200.ops.weights import mark_shadow_fresh, set_bf16_shadow

EXPERT_SUFFIXES = (".experts_gate_weights", ".experts_up_weights", ".experts_down_weights")


class FlatParams:
    def __init__(self, model: torch.nn.Module, align: int = 64, pad_to_multiple: int = 1, with_bf16: bool = True,
                 heap_factory=None):
        """``heap_factory(nbytes)`` (optional) returns a :class:`~tinytron_b200.parallel.symm.SymmetricHeap`
        of at least ``nbytes`` from which the three flat buffers are carved, so peers can
        reduce-scatter the gradients and all-gather the parameters with NVLink loads and
        stores (every rank builds the same layout, so offsets match across ranks)."""
        named = []
        seen = set()
        for name, p in model.named_parameters():
            if id(p) in seen or not p.requires_grad:
                continue
            seen.add(id(p))
            named.append((name, p))
        dense = [(n, p) for n, p in named if not n.endswith(EXPERT_SUFFIXES)]
        expert = [(n, p) for n, p in named if n.endswith(EXPERT_SUFFIXES)]
        self.named = dense + expert
        self.params = [p for _, p in self.named]
        self.names = [n for n, _ in self.named]
        offsets, off = [], 0
        for _, p in self.named:
            off = (off + align - 1) // align * align
            offsets.append(off)
            off += p.numel()
        total = (off + align - 1) // align * align
        total = (total + pad_to_multiple - 1) // pad_to_multiple * pad_to_multiple
        self.dense_numel = offsets[len(dense)] if expert else total
        self.numel = total
        self.offsets = offsets
        device = self.params[0].device
        self.device = device
        self.heap = None
        if heap_factory is not None:
            from .symm import SymmetricHeap

            specs = [(total, torch.float32), (total, torch.float32)] + ([(total, torch.bfloat16)] if with_bf16 else [])
            self.heap = heap_factory(SymmetricHeap.bytes_needed(*specs))
            self.data = self.heap.alloc(total, torch.float32)
            self.grad = self.heap.alloc(total, torch.float32)
            self.bf16 = self.heap.alloc(total, torch.bfloat16) if with_bf16 else None
        else:
            self.data = torch.zeros(total, dtype=torch.float32, device=device)
            self.grad = torch.zeros(total, dtype=torch.float32, device=device)
            self.bf16 = torch.zeros(total, dtype=torch.bfloat16, device=device) if with_bf16 else None
        for (name, p), o in zip(self.named, offsets):
            n = p.numel()
            view = self.data[o:o + n].view_as(p)
            view.copy_(p.data)
            p.data = view
            p.__dict__["main_grad"] = self.grad[o:o + n].view_as(p)
            if self.bf16 is not None:
                set_bf16_shadow(p, self.bf16[o:o + n].view_as(p))

    def param_slice(self, p: torch.Tensor) -> tuple[int, int]:
        i = next(i for i, q in enumerate(self.params) if q is p)
        return self.offsets[i], self.offsets[i] + p.numel()

    def zero_grad(self) -> None:
        self.grad.zero_()

    @torch.no_grad()
    def refresh_bf16(self) -> None:
        if self.bf16 is not None:
            self.bf16.copy_(self.data)
            for p in self.params:
                mark_shadow_fresh(p)

    def mark_shadows_fresh(self) -> None:
        for p in self.params:
            mark_shadow_fresh(p)

    def expose_grads(self) -> None:
        """Point ``p.grad`` at the main_grad views (API compatibility, no copy)."""
        for p in self.params:
            p.grad = p.__dict__["main_grad"]
