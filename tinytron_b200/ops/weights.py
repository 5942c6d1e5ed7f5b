"""Weight views used by the CUDA path.

Master weights are fp32 ``nn.Parameter`` objects (the reference trains fp32
masters under bf16 autocast, trainer.py:330-337).  The tensor-core GEMMs consume a
bf16 *shadow* of each weight and accumulate weight gradients straight into an fp32
``main_grad`` buffer inside the GEMM epilogue, instead of autocast re-casting every
weight on every forward and autograd materialising separate fp32 grads.

* ``bf16_of(p)`` returns the bf16 shadow, refreshing it when the parameter's
  version counter says the fp32 master changed (e.g. ``load_state_dict``).  The
  fused optimizer kernels write master and shadow together, so no refresh is
  needed after an optimizer step.
* ``main_grad`` is attached by :class:`tinytron_b200.parallel.buffers.FlatParams`;
  without it, weight grads are returned to autograd as ordinary fp32 ``.grad``.
"""
from __future__ import annotations

import torch


def bf16_of(p: torch.Tensor) -> torch.Tensor:
    d = p.__dict__
    shadow = d.get("_tt_bf16")
    ver = p._version
    if shadow is None:
        shadow = p.detach().to(torch.bfloat16)
        d["_tt_bf16"] = shadow
        d["_tt_bf16_ver"] = ver
    elif d.get("_tt_bf16_ver") != ver:
        with torch.no_grad():
            shadow.copy_(p.detach())
        d["_tt_bf16_ver"] = ver
    return shadow


def set_bf16_shadow(p: torch.Tensor, shadow: torch.Tensor) -> None:
    """Attach an externally owned bf16 view (e.g. a slice of a flat buffer) and fill it."""
    with torch.no_grad():
        shadow.copy_(p.detach())
    p.__dict__["_tt_bf16"] = shadow
    p.__dict__["_tt_bf16_ver"] = p._version


def mark_shadow_fresh(p: torch.Tensor) -> None:
    """Record that the shadow matches the master (after a fused optimizer update)."""
    p.__dict__["_tt_bf16_ver"] = p._version


def main_grad_of(p: torch.Tensor):
    return p.__dict__.get("main_grad")


def adjacent_views(tensors: list[torch.Tensor]) -> bool:
    """True when the tensors are back-to-back contiguous views of one storage."""
    if not tensors or any(t is None for t in tensors):
        return False
    if any(not t.is_contiguous() for t in tensors):
        return False
    st = tensors[0].untyped_storage().data_ptr()
    nxt = tensors[0].data_ptr() + tensors[0].numel() * tensors[0].element_size()
    for t in tensors[1:]:
        if t.untyped_storage().data_ptr() != st or t.data_ptr() != nxt:
            return False
        nxt = t.data_ptr() + t.numel() * t.element_size()
    return True


def concat_rows(tensors: list[torch.Tensor]) -> torch.Tensor:
    """[sum(rows), cols] view when adjacent, else a concatenated copy."""
    if adjacent_views(tensors):
        first = tensors[0]
        rows = sum(t.shape[0] for t in tensors)
        return first.as_strided((rows,) + tuple(first.shape[1:]), first.stride())
    return torch.cat(tensors, 0)


def notify_grad_ready(params) -> None:
    """Tell the gradient reducer (if any) that these params' main_grad are final for
    this backward.  Set by FlatParams.attach_reducer."""
    for p in params:
        cb = p.__dict__.get("_tt_grad_ready")
        if cb is not None:
            cb(p)


def concat_rows_cached(owner: torch.Tensor, key: str, tensors: list[torch.Tensor]) -> torch.Tensor:
    """:func:`concat_rows`, but when a copy is needed (the tensors are not adjacent, e.g.
    separate bf16 shadows outside a flat buffer) the copy is kept on ``owner`` and reused
    while every source tensor keeps its storage and version (weights at inference)."""
    if adjacent_views(tensors):
        return concat_rows(tensors)
    d = owner.__dict__
    stamp = tuple((t.data_ptr(), t._version) for t in tensors)
    hit = d.get(key)
    if hit is not None and hit[0] == stamp:
        return hit[1]
    out = torch.cat(tensors, 0)
    d[key] = (stamp, out)
    return out
