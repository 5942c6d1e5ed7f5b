"""Ulysses sequence parallelism (reference: tinytron/distributed/sequence_parallel/ulysses.py:7-86).

``ulysses_all_to_all``: autograd all-to-all over dim 0 (equal splits), identical in
forward and backward.  ``allreduce_non_expert_grads_across_sp``: SUM all-reduce of
non-expert gradients across the SP group (reference semantics: sum, not mean),
bucketed; it reduces ``main_grad`` buffers when the model uses flat fp32 grads.

The attention module uses :func:`route_heads_to_ranks` / :func:`gather_heads_from_ranks`
(head<->sequence transposes with *unexpanded* GQA routing: a kv head is sent only to
the ranks whose q heads read it, instead of expanding kv to Hq heads first).  On CUDA
inside one node both run as fused pack / exchange kernels on a symmetric heap
(``csrc/runtime/ulysses.cu``): the routing and the layout changes happen inside the
kernels that move the data, so no stacked, permuted or expanded copy is ever made.
"""
from __future__ import annotations

import torch
import torch.distributed as dist


def _a2a(x: torch.Tensor, group) -> torch.Tensor:
    """Equal-split all-to-all on dim 0: the symmetric-heap kernel (peer loads) when
    enabled for the group and the chunks are 16-byte multiples, else NCCL."""
    from .symm import heap_all_to_all_for

    a = heap_all_to_all_for(group) if x.is_cuda else None
    if a is not None and (x.numel() * x.element_size()) % (16 * x.shape[0]) == 0:
        slot = a.slot(x.shape, x.dtype)
        slot.copy_(x)
        return a.exchange(slot)
    x = x.contiguous()
    out = torch.empty_like(x)
    dist.all_to_all_single(out, x, group=group)
    return out


class UlyssesAllToAll(torch.autograd.Function):
    @staticmethod
    def forward(ctx, input_tensor, sp_group):
        ctx.sp_group = sp_group
        return _a2a(input_tensor, sp_group)

    @staticmethod
    def backward(ctx, grad_output):
        return _a2a(grad_output, ctx.sp_group), None


def ulysses_all_to_all(input_tensor: torch.Tensor, sp_group) -> torch.Tensor:
    return UlyssesAllToAll.apply(input_tensor, sp_group)


def kv_heads_for_rank(rank: int, sp: int, Hq: int, Hkv: int) -> tuple[int, int]:
    """[start, end) of kv heads read by the q heads rank `rank` owns after the transpose."""
    hq_l = Hq // sp
    G = Hq // Hkv
    return (rank * hq_l) // G, (rank * hq_l + hq_l - 1) // G + 1


def native_gqa_routing(sp: int, Hq: int, Hkv: int) -> bool:
    """True when each rank's q heads map onto its kv heads with the kernel's uniform
    h_local // (Hq_l / Hkv_l) rule (so kv heads are sent unexpanded)."""
    if Hq % sp:
        return False
    hq_l, G = Hq // sp, Hq // Hkv
    if Hkv % sp == 0:
        return True
    return G % hq_l == 0  # every rank's q heads fall inside one kv group


# ----------------------------------------------------------------------------- fused kernels
def _C():
    from tinytron_b200.ops import _ext

    return _ext.load()


def _kv_starts(sp: int, Hq: int, Hkv: int) -> list[int]:
    return [kv_heads_for_rank(r, sp, Hq, Hkv)[0] for r in range(sp)]


class _FusedHeadsFn(torch.autograd.Function):
    """q|k|v of this rank's tokens -> this rank's heads over the full sequence, by the
    fused pack / exchange kernels (the GQA routing and both layout changes are inside
    the kernels; no intermediate tensors)."""

    @staticmethod
    def forward(ctx, qkv, ex, B, T, Hq, Hkv, D, sp, hq_l, hkv_l):
        W = (hq_l + 2 * hkv_l) * D
        kv0 = _kv_starts(sp, Hq, Hkv)
        gid, off, sb = ex.ensure(sp * B * T * W * 2)
        C = _C()
        C.ul_pack(gid, off, sb, qkv, B, T, [T, 0, 1], W, hq_l * D, (hq_l + hkv_l) * D,
                  [c * hq_l * D for c in range(sp)], [Hq * D + k * D for k in kv0],
                  [(Hq + Hkv) * D + k * D for k in kv0])
        full = torch.empty(B * sp * T, W, device=qkv.device, dtype=torch.bfloat16)
        C.ul_exchange(gid, off, sb, full, B, T, [sp * T, T, 1], 0, W)
        ctx.cfg = (ex, B, T, Hq, Hkv, D, sp, hq_l, hkv_l, kv0)
        return full

    @staticmethod
    def backward(ctx, g_full):
        ex, B, T, Hq, Hkv, D, sp, hq_l, hkv_l, kv0 = ctx.cfg
        W = (hq_l + 2 * hkv_l) * D
        g_full = g_full.to(torch.bfloat16).contiguous()
        gid, off, sb = ex.ensure(sp * B * T * W * 2)
        C = _C()
        C.ul_pack(gid, off, sb, g_full, B, T, [sp * T, T, 1], W, W, W, [0] * sp, [0] * sp, [0] * sp)
        dqkv = torch.empty(B * T, (Hq + 2 * Hkv) * D, device=g_full.device, dtype=torch.bfloat16)
        C.ul_exchange_qkv_grad(gid, off, sb, dqkv, B, T, Hq, Hkv, D, hq_l, hkv_l, kv0)
        return dqkv, None, None, None, None, None, None, None, None, None


class _FusedTokensFn(torch.autograd.Function):
    """Attention output of this rank's heads over the full sequence -> all heads of this
    rank's tokens (the c_proj input layout), by the fused pack / exchange kernels."""

    @staticmethod
    def forward(ctx, o, ex, B, T, Hq, D, sp):
        hq_l = Hq // sp
        W = hq_l * D
        gid, off, sb = ex.ensure(sp * B * T * W * 2)
        C = _C()
        C.ul_pack(gid, off, sb, o, B, T, [sp * T, T, 1], W, W, W, [0] * sp, [0] * sp, [0] * sp)
        y = torch.empty(B * T, Hq * D, device=o.device, dtype=torch.bfloat16)
        C.ul_exchange(gid, off, sb, y, B, T, [T, 0, 1], W, W)
        ctx.cfg = (ex, B, T, Hq, D, sp)
        return y

    @staticmethod
    def backward(ctx, g_y):
        ex, B, T, Hq, D, sp = ctx.cfg
        hq_l = Hq // sp
        W = hq_l * D
        g_y = g_y.to(torch.bfloat16).contiguous()
        gid, off, sb = ex.ensure(sp * B * T * W * 2)
        C = _C()
        C.ul_pack(gid, off, sb, g_y, B, T, [T, 0, 1], W, W, W, [c * W for c in range(sp)], [0] * sp, [0] * sp)
        do = torch.empty(B * sp * T, W, device=g_y.device, dtype=torch.bfloat16)
        C.ul_exchange(gid, off, sb, do, B, T, [sp * T, T, 1], 0, W)
        return do, None, None, None, None, None, None


def _fused_ok(x: torch.Tensor, group, sp: int, Hq: int, Hkv: int, D: int):
    if not x.is_cuda or x.dtype != torch.bfloat16 or sp > 8 or D % 8:
        return None
    if not native_gqa_routing(sp, Hq, Hkv):
        return None
    from .symm import ulysses_exchange_for

    return ulysses_exchange_for(group)


def route_heads_to_ranks(qkv: torch.Tensor, B: int, T_loc: int, Hq: int, Hkv: int, D: int, sp: int, group):
    """qkv [B*T_loc, (Hq+2Hkv)*D] (this rank's sequence chunk, all heads) ->
    [B*T_full, (Hq_l + 2*Hkv_l)*D] (full sequence, this rank's heads)."""
    hq_l = Hq // sp
    ex = _fused_ok(qkv, group, sp, Hq, Hkv, D)
    if ex is not None:
        k0, k1 = kv_heads_for_rank(0, sp, Hq, Hkv)
        hkv_l = k1 - k0
        full = _FusedHeadsFn.apply(qkv.contiguous(), ex, B, T_loc, Hq, Hkv, D, sp, hq_l, hkv_l)
        return full, hq_l, hkv_l
    x = qkv.view(B, T_loc, Hq + 2 * Hkv, D)
    if native_gqa_routing(sp, Hq, Hkv):
        parts = []
        for r in range(sp):
            k0, k1 = kv_heads_for_rank(r, sp, Hq, Hkv)
            parts.append(torch.cat([x[:, :, r * hq_l:(r + 1) * hq_l], x[:, :, Hq + k0:Hq + k1],
                                    x[:, :, Hq + Hkv + k0:Hq + Hkv + k1]], dim=2))
        hkv_l = parts[0].shape[2] - hq_l
        hkv_l //= 2
    else:  # expand kv to Hq heads (reference behaviour) when routing is not uniform
        G = Hq // Hkv
        k = x[:, :, Hq:Hq + Hkv].repeat_interleave(G, dim=2)
        v = x[:, :, Hq + Hkv:].repeat_interleave(G, dim=2)
        parts = [torch.cat([x[:, :, r * hq_l:(r + 1) * hq_l], k[:, :, r * hq_l:(r + 1) * hq_l],
                            v[:, :, r * hq_l:(r + 1) * hq_l]], dim=2) for r in range(sp)]
        hkv_l = hq_l
    send = torch.stack(parts, 0)  # [sp, B, T_loc, W_l/D, D]
    recv = ulysses_all_to_all(send, group)  # [sp(src chunk), B, T_loc, ...]
    full = recv.permute(1, 0, 2, 3, 4).reshape(B * sp * T_loc, (hq_l + 2 * hkv_l) * D)
    return full, hq_l, hkv_l


def gather_heads_from_ranks(o: torch.Tensor, B: int, T_loc: int, Hq: int, D: int, sp: int, group) -> torch.Tensor:
    """o [B*T_full, Hq_l*D] (full sequence, local heads) -> [B, T_loc, Hq*D] (local chunk, all heads)."""
    hq_l = Hq // sp
    ex = _fused_ok(o, group, sp, Hq, Hq, D)
    if ex is not None:
        return _FusedTokensFn.apply(o.contiguous(), ex, B, T_loc, Hq, D, sp).view(B, T_loc, Hq * D)
    send = o.view(B, sp, T_loc, hq_l * D).permute(1, 0, 2, 3).contiguous()  # [dst chunk, B, T_loc, hq_l*D]
    recv = ulysses_all_to_all(send, group)  # [src rank (head block), B, T_loc, hq_l*D]
    return recv.permute(1, 2, 0, 3).reshape(B, T_loc, Hq * D)


@torch.no_grad()
def allreduce_non_expert_grads_across_sp(model, sp_group, sp_world_size: int,
                                         expert_local_param_suffixes: tuple[str, ...], bucket_size_mb: int = 400):
    """SUM-all-reduce every non-expert gradient across the SP group, in flat buckets."""
    if sp_world_size <= 1:
        return
    grads: dict[tuple, list[torch.Tensor]] = {}
    seen = set()
    for name, p in model.named_parameters():
        if id(p) in seen or name.endswith(expert_local_param_suffixes):
            continue
        seen.add(id(p))
        g = p.__dict__.get("main_grad")
        if g is None:
            g = p.grad
        if g is None:
            continue
        grads.setdefault((g.device, g.dtype), []).append(g)
    limit = max(1, bucket_size_mb) * 1024 * 1024
    for tensors in grads.values():
        bucket, size = [], 0
        for t in tensors + [None]:
            if t is None or (bucket and size + t.numel() * t.element_size() > limit):
                if bucket:
                    flat = torch.cat([b.reshape(-1) for b in bucket])
                    dist.all_reduce(flat, op=dist.ReduceOp.SUM, group=sp_group)
                    off = 0
                    for b in bucket:
                        b.copy_(flat[off:off + b.numel()].view_as(b))
                        off += b.numel()
                bucket, size = [], 0
            if t is not None:
                bucket.append(t)
                size += t.numel() * t.element_size()
