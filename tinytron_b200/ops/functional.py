"""Autograd functions for the sm_100a path.  Every op here launches the in-tree
CUDA extension (no PyTorch/cuBLAS fallback on the GPU); see ``tinytron_b200.ops``
for the device dispatch and the CPU reference path.

Dtype contract (matches the reference's fp32-master + bf16-autocast numerics):
  * residual stream, norms, embedding table, master weights, weight grads: fp32
  * projection inputs/outputs, attention operands, logits: bf16
  * weight gradients accumulate in fp32 inside the GEMM epilogue.
"""
from __future__ import annotations

import math
import os

import torch

from . import _ext
from .rope import rope_tables
from .weights import adjacent_views, bf16_of, concat_rows, concat_rows_cached, main_grad_of, notify_grad_ready


def C():
    return _ext.load()


def _bf16(x: torch.Tensor) -> torch.Tensor:
    x = x if x.dtype == torch.bfloat16 else x.to(torch.bfloat16)
    return x if x.is_contiguous() else x.contiguous()


# ----------------------------------------------------------------------------- GEMM helpers
# Decode-sized products (<= 32 token rows) against a large weight run on the
# weight-streaming split-K kernel (csrc/gemm/skinny.cu); TT_SKINNY=0 keeps them on the
# tile GEMM (for comparisons).
SKINNY_MAX_ROWS = 32
_SKINNY_MIN_WEIGHT = 1 << 21  # weight elements (4 MB in bf16)


def skinny_enabled() -> bool:
    return os.environ.get("TT_SKINNY", "1") != "0"


def gemm_nt(a: torch.Tensor, w16: torch.Tensor, out_dtype=torch.bfloat16) -> torch.Tensor:
    """a [M, K] @ w16[N, K]^T."""
    out = torch.empty(a.shape[0], w16.shape[0], device=a.device, dtype=out_dtype)
    if (out_dtype == torch.bfloat16 and a.shape[0] <= SKINNY_MAX_ROWS and w16.numel() >= _SKINNY_MIN_WEIGHT
            and w16.shape[0] % 4 == 0 and skinny_enabled()):
        C().skinny_linear(a, w16, out)
    else:
        C().gemm(a, w16, out, False, False, False, 1.0, None, 0)
    return out


@torch.no_grad()
def linear_row_parallel(x: torch.Tensor, w16: torch.Tensor, ar) -> torch.Tensor | None:
    """x [..., K] @ w16[N, K]^T summed over the SEP group whose graph-safe heap all-reduce
    is ``ar`` (inference): the decode-sized product's split-sum kernel writes its result
    straight into ``ar``'s slot and signals the peers, so only the reducing kernel follows
    (no separate publish copy).  None when the shape does not take this path."""
    x2d = _bf16(x.reshape(-1, x.shape[-1]))
    M, N = x2d.shape[0], w16.shape[0]
    if M > SKINNY_MAX_ROWS or N % 4 or not skinny_enabled() or not ar.fits(M * N):
        return None
    out = torch.empty(M, N, device=x.device, dtype=torch.bfloat16)
    C().skinny_linear(x2d, w16, out, *ar.publish_target())
    ar.reduce_into(out)
    return out.view(*x.shape[:-1], N)


def gemm_nn(a: torch.Tensor, w16: torch.Tensor, alpha_t=None) -> torch.Tensor:
    """a [M, N] @ w16[N, K]  (dgrad)."""
    out = torch.empty(a.shape[0], w16.shape[1], device=a.device, dtype=torch.bfloat16)
    C().gemm(a, w16, out, False, True, False, 1.0, alpha_t, 0)
    return out


def weight_grads(weights, dy2d: torch.Tensor, x2d: torch.Tensor, alpha_t=None):
    """Gradients of y = x @ cat(weights)^T w.r.t. each weight: dW = dy^T x.

    Accumulates into ``main_grad`` (one GEMM when the main grads are adjacent) and
    returns Nones, or returns fresh fp32 grads for autograd when there is no main_grad.
    """
    mgs = [main_grad_of(w) for w in weights]
    if all(m is not None for m in mgs):
        if len(mgs) == 1 or adjacent_views(mgs):
            C().gemm(dy2d, x2d, concat_rows(mgs), True, True, True, 1.0, alpha_t, 0)
        else:
            tmp = torch.empty(dy2d.shape[1], x2d.shape[1], device=dy2d.device, dtype=torch.float32)
            C().gemm(dy2d, x2d, tmp, True, True, False, 1.0, alpha_t, 0)
            r = 0
            for m in mgs:
                m.add_(tmp[r:r + m.shape[0]])
                r += m.shape[0]
        notify_grad_ready(weights)
        return [None] * len(weights)
    tmp = torch.empty(dy2d.shape[1], x2d.shape[1], device=dy2d.device, dtype=torch.float32)
    C().gemm(dy2d, x2d, tmp, True, True, False, 1.0, alpha_t, 0)
    out, r = [], 0
    for w in weights:
        out.append(tmp[r:r + w.shape[0]].view_as(w))
        r += w.shape[0]
    return out


# ----------------------------------------------------------------------------- Linear
class LinearFn(torch.autograd.Function):
    """y = x @ cat(weights)^T  (several weights sharing an input are fused into one GEMM)."""

    @staticmethod
    def forward(ctx, x, *weights):
        shape = x.shape
        x2d = _bf16(x.reshape(-1, shape[-1]))
        w16 = concat_rows_cached(weights[0], "_tt_cat", [bf16_of(w) for w in weights]) if len(weights) > 1 \
            else bf16_of(weights[0])
        y = gemm_nt(x2d, w16)
        ctx.save_for_backward(x2d, w16)
        ctx.weights = weights
        ctx.in_shape = shape
        ctx.x_dtype = x.dtype
        return y.view(*shape[:-1], w16.shape[0])

    @staticmethod
    def backward(ctx, dy):
        x2d, w16 = ctx.saved_tensors
        dy2d = _bf16(dy.reshape(-1, dy.shape[-1]))
        dx = None
        if ctx.needs_input_grad[0]:
            dx = gemm_nn(dy2d, w16).view(ctx.in_shape)
            if ctx.x_dtype != torch.bfloat16:
                dx = dx.to(ctx.x_dtype)
        grads = weight_grads(ctx.weights, dy2d, x2d)
        return (dx, *grads)


# ----------------------------------------------------------------------------- SwiGLU MLP
class SwiGLUMLPFn(torch.autograd.Function):
    """down(silu(gate(x)) * up(x)); gate|up run as one tcgen05 GEMM with the SwiGLU
    epilogue, the backward's SwiGLU derivative runs in the down-proj dgrad epilogue."""

    @staticmethod
    def forward(ctx, x, w_gate, w_up, w_down):
        shape = x.shape
        x2d = _bf16(x.reshape(-1, shape[-1]))
        M = x2d.shape[0]
        w_gu = concat_rows_cached(w_gate, "_tt_gu_cat", [bf16_of(w_gate), bf16_of(w_up)])
        wd = bf16_of(w_down)
        I = w_gate.shape[0]
        act = torch.empty(M, I, device=x.device, dtype=torch.bfloat16)
        gu = torch.empty(M, 2 * I, device=x.device, dtype=torch.bfloat16)
        C().gemm_swiglu(x2d, w_gu, act, gu)
        y = gemm_nt(act, wd)
        ctx.save_for_backward(x2d, act, gu, w_gu, wd)
        ctx.weights = (w_gate, w_up, w_down)
        ctx.in_shape = shape
        return y.view(*shape[:-1], wd.shape[0])

    @staticmethod
    def backward(ctx, dy):
        x2d, act, gu, w_gu, wd = ctx.saved_tensors
        w_gate, w_up, w_down = ctx.weights
        dy2d = _bf16(dy.reshape(-1, dy.shape[-1]))
        dgu = torch.empty_like(gu)
        C().gemm_dswiglu(dy2d, wd, gu, dgu, 1.0)
        (g_down,) = weight_grads([w_down], dy2d, act)
        dx = gemm_nn(dgu, w_gu).view(ctx.in_shape)
        g_gate, g_up = weight_grads([w_gate, w_up], dgu, x2d)
        return dx, g_gate, g_up, g_down


# ----------------------------------------------------------------------------- MoE
class RouterTopKFn(torch.autograd.Function):
    """Router top-k + softmax over the selected logits (one warp per token)."""

    @staticmethod
    def forward(ctx, logits, k):
        l2d = logits.reshape(-1, logits.shape[-1]).contiguous()
        N = l2d.shape[0]
        w = torch.empty(N, k, device=logits.device, dtype=torch.float32)
        sel = torch.empty(N, k, device=logits.device, dtype=torch.int32)
        C().moe_topk_softmax(l2d, k, w, sel)
        ctx.save_for_backward(w, sel)
        ctx.shape = logits.shape
        ctx.dtype = l2d.dtype
        ctx.mark_non_differentiable(sel)
        return w.view(*logits.shape[:-1], k), sel.view(*logits.shape[:-1], k)

    @staticmethod
    def backward(ctx, dw, _dsel):
        w, sel = ctx.saved_tensors
        dl = torch.empty(w.shape[0], ctx.shape[-1], device=w.device, dtype=ctx.dtype)
        C().moe_topk_softmax_bwd(dw.reshape(w.shape).float().contiguous(), w, sel, dl)
        return dl.view(ctx.shape), None


def _expert_grad(param, shape2d):
    """fp32 gradient target of an expert weight viewed as [E*rows, cols]: its main_grad
    (accumulated) or a fresh buffer returned to autograd."""
    mg = main_grad_of(param)
    if mg is not None:
        return mg.view(shape2d), True
    return torch.zeros(shape2d, device=param.device, dtype=torch.float32), False


# Expert segments start on 256-row boundaries when experts average at least 256 rows
# (training), so the CTA-pair kernel (256-row tiles) can run the grouped GEMMs; with few
# rows per expert (decode) 128-row segments halve the padding and the single-CTA kernel runs.
def moe_align(pairs: int, experts: int) -> int:
    return 256 if pairs >= 256 * experts else 128


@torch.no_grad()
def moe_experts_decode(x, sel, weights, w_gate, w_up, w_down, e_lo: int | None = None, out=None, publish=None):
    """Routed experts for a decode-sized batch (<= 32 tokens, no autograd) on the
    weight-streaming kernels: every expert's weights are read once by all SMs, token rows
    sit in unpadded expert segments, and the down projection's split sums are combined
    with the top-k weights in one pass.  ``e_lo`` set: only the experts [e_lo, e_lo + E)
    held by this rank (the others' pairs go to an extra segment that is never computed),
    as in :func:`moe_experts_local`.  ``publish`` (a graph-safe heap all-reduce of the EP
    group): the combine writes the partial sums into its slot and signals the peers, and
    the returned tensor is already the sum over the group."""
    x2d = _bf16(x.reshape(-1, x.shape[-1]))
    N, H = x2d.shape
    E, I = w_gate.shape[0], w_gate.shape[1]
    k = sel.shape[-1]
    c = C()
    dev = x.device
    ids = sel.reshape(-1).to(torch.int32).contiguous()
    groups = E if e_lo is None else E + 1  # + the never-computed group of other ranks' pairs
    P = ids.numel()
    cap = c.moe_row_capacity(P, groups, 1)
    grp_off = torch.empty(groups + 1, device=dev, dtype=torch.int32)
    slot = torch.empty(P, device=dev, dtype=torch.int32)
    row_pair = torch.empty(cap, device=dev, dtype=torch.int32)
    c.moe_layout(ids, groups, grp_off, slot, row_pair, 1, -1 if e_lo is None else int(e_lo))
    g_loc = grp_off[:E + 1]
    xr = torch.empty(cap, H, device=dev, dtype=torch.bfloat16)
    c.moe_gather_rows(x2d, row_pair, g_loc, k, xr)
    w_gu = concat_rows_cached(w_gate, "_tt_gu_cat", [bf16_of(w_gate).view(E * I, H), bf16_of(w_up).view(E * I, H)])
    act = torch.empty(cap, I, device=dev, dtype=torch.bfloat16)
    c.moe_skinny_swiglu(xr, w_gu, g_loc, E, act)
    out = torch.empty(N, H, device=dev, dtype=torch.bfloat16) if out is None else out
    w32 = weights.reshape(-1).float().contiguous() if weights is not None else None
    target = publish.publish_target() if publish is not None else (-1, 0, 0)
    c.moe_skinny_down_combine(act, bf16_of(w_down).view(E * H, I), g_loc, E, slot, w32, k, out, g_loc[E:E + 1],
                              *target)
    if publish is not None:
        publish.reduce_into(out)
    return out


def moe_experts_local(x, sel, weights, w_gate, w_up, w_down, e_lo: int, out=None, publish=None):
    """Expert-parallel inference: the weighted partial sum over the experts
    [e_lo, e_lo + E_local) held by this rank, for every token (zeros where none of a
    token's experts is here).  Everything stays on the device (no host synchronisation,
    so a decode step containing it can be captured in a CUDA graph): pairs routed
    elsewhere go to an extra "remote" segment that the grouped GEMMs never compute, and
    the combine stops at the local row count read on the device.  Returns (output,
    reduced): with ``publish`` (the EP group's heap all-reduce) a decode-sized batch is
    summed over the group by the fused publish (reduced True); otherwise the caller
    all-reduces the partial sums."""
    N = x.reshape(-1, x.shape[-1]).shape[0]
    if N <= SKINNY_MAX_ROWS and skinny_enabled():
        if publish is not None and not publish.fits(N * x.shape[-1]):
            publish = None
        return moe_experts_decode(x, sel, weights, w_gate, w_up, w_down, e_lo, out, publish), publish is not None
    x2d = _bf16(x.reshape(-1, x.shape[-1]))
    N, H = x2d.shape
    E, I = w_gate.shape[0], w_gate.shape[1]
    k = sel.shape[-1]
    c = C()
    dev = x.device
    local = sel.reshape(-1).to(torch.int32).contiguous()
    P = local.numel()
    align = moe_align(P, E + 1)
    pair = align == 256
    cap = c.moe_row_capacity(P, E + 1, align)
    grp_off = torch.empty(E + 2, device=dev, dtype=torch.int32)
    slot = torch.empty(P, device=dev, dtype=torch.int32)
    row_pair = torch.empty(cap, device=dev, dtype=torch.int32)
    c.moe_layout(local, E + 1, grp_off, slot, row_pair, align, int(e_lo))
    g_loc = grp_off[:E + 1]  # local expert segments; g_loc[E] = rows computed on this rank
    xr = torch.empty(cap, H, device=dev, dtype=torch.bfloat16)
    c.moe_gather_rows(x2d, row_pair, g_loc, k, xr)
    w_gu = concat_rows_cached(w_gate, "_tt_gu_cat", [bf16_of(w_gate).view(E * I, H), bf16_of(w_up).view(E * I, H)])
    act = torch.empty(cap, I, device=dev, dtype=torch.bfloat16)
    gu = torch.empty(cap, 2 * I, device=dev, dtype=torch.bfloat16)
    c.moe_gemm_swiglu(xr, w_gu, act, gu, g_loc, E, pair)
    yr = torch.empty(cap, H, device=dev, dtype=torch.bfloat16)
    c.moe_gemm(act, bf16_of(w_down).view(E * H, I), yr, g_loc, E, False, H, 0, 0, pair)
    out = torch.empty(N, H, device=dev, dtype=torch.bfloat16) if out is None else out
    w32 = weights.reshape(-1).float().contiguous() if weights is not None else None
    c.moe_combine(yr, slot, w32, k, out, grp_off[E:E + 1])
    return out, False


class MoEExpertsFn(torch.autograd.Function):
    """Routed SwiGLU experts on grouped tcgen05 GEMMs.

    Token rows are laid out by expert in 128-row-aligned segments on the device
    (``moe_layout``); gate|up run as one grouped GEMM with the SwiGLU epilogue, the
    down projection as a second one, and the top-k weighted sum in ``moe_combine``.
    Backward: combine -> (dy_rows, dweights); down dgrad with the SwiGLU backward in its
    epilogue; gate|up dgrad over the stacked weights; per-expert weight gradients
    reduce over each expert's token segment straight into the fp32 main grads.
    """

    @staticmethod
    def forward(ctx, x, sel, weights, w_gate, w_up, w_down):
        shape = x.shape
        x2d = _bf16(x.reshape(-1, shape[-1]))
        N, H = x2d.shape
        E, I = w_gate.shape[0], w_gate.shape[1]
        k = sel.shape[-1]
        c = C()
        sel32 = sel.reshape(-1).to(torch.int32).contiguous()
        P = sel32.numel()
        align = moe_align(P, E)
        pair = align == 256
        cap = c.moe_row_capacity(P, E, align)
        dev = x.device
        grp_off = torch.empty(E + 1, device=dev, dtype=torch.int32)
        slot = torch.empty(P, device=dev, dtype=torch.int32)
        row_pair = torch.empty(cap, device=dev, dtype=torch.int32)
        c.moe_layout(sel32, E, grp_off, slot, row_pair, align)
        xr = torch.empty(cap, H, device=dev, dtype=torch.bfloat16)
        c.moe_gather_rows(x2d, row_pair, grp_off, k, xr)
        w_gu = concat_rows_cached(w_gate, "_tt_gu_cat", [bf16_of(w_gate).view(E * I, H), bf16_of(w_up).view(E * I, H)])
        wd = bf16_of(w_down).view(E * H, I)
        act = torch.empty(cap, I, device=dev, dtype=torch.bfloat16)
        gu = torch.empty(cap, 2 * I, device=dev, dtype=torch.bfloat16)
        c.moe_gemm_swiglu(xr, w_gu, act, gu, grp_off, E, pair)
        yr = torch.empty(cap, H, device=dev, dtype=torch.bfloat16)
        c.moe_gemm(act, wd, yr, grp_off, E, False, H, 0, 0, pair)
        w32 = weights.reshape(-1).float().contiguous() if weights is not None else None
        out = torch.empty(N, H, device=dev, dtype=torch.bfloat16)
        c.moe_combine(yr, slot, w32, k, out)
        ctx.save_for_backward(xr, act, gu, yr, grp_off, slot, row_pair, w_gu, wd)
        ctx.w32 = w32
        ctx.params = (w_gate, w_up, w_down)
        ctx.dims = (N, H, E, I, k, cap)
        ctx.pair = pair
        ctx.shape = shape
        ctx.has_w = weights is not None
        return out.view(shape)

    @staticmethod
    def backward(ctx, dout):
        xr, act, gu, yr, grp_off, slot, row_pair, w_gu, wd = ctx.saved_tensors
        w_gate, w_up, w_down = ctx.params
        N, H, E, I, k, cap = ctx.dims
        c = C()
        dev = xr.device
        d2d = _bf16(dout.reshape(N, H))
        w32 = ctx.w32 if ctx.has_w else torch.ones(N * k, device=dev, dtype=torch.float32)
        dyr = torch.empty(cap, H, device=dev, dtype=torch.bfloat16)
        dw = torch.empty(N * k, device=dev, dtype=torch.float32)
        c.moe_combine_bwd(d2d, yr, row_pair, w32, grp_off, k, dyr, dw)
        dgu = torch.empty(cap, 2 * I, device=dev, dtype=torch.bfloat16)
        c.moe_gemm_dswiglu(dyr, wd, gu, dgu, grp_off, E, ctx.pair)
        g_down, main_d = _expert_grad(w_down, (E * H, I))
        c.moe_gemm_wgrad(dyr, act, g_down, grp_off, E, True, True)
        dxr = torch.empty(cap, H, device=dev, dtype=torch.bfloat16)
        c.moe_gemm(dgu, w_gu, dxr, grp_off, E, True, I, I, E * I, ctx.pair)
        g_gate, main_g = _expert_grad(w_gate, (E * I, H))
        g_up, main_u = _expert_grad(w_up, (E * I, H))
        c.moe_gemm_wgrad(dgu[:, :I], xr, g_gate, grp_off, E, True, True)
        c.moe_gemm_wgrad(dgu[:, I:], xr, g_up, grp_off, E, True, True)
        dx = torch.empty(N, H, device=dev, dtype=torch.bfloat16)
        c.moe_combine(dxr, slot, None, k, dx)
        notify_grad_ready([p for p, m in ((w_gate, main_g), (w_up, main_u), (w_down, main_d)) if m])
        return (dx.view(ctx.shape), None, dw.view(N, k) if ctx.has_w else None,
                None if main_g else g_gate.view_as(w_gate), None if main_u else g_up.view_as(w_up),
                None if main_d else g_down.view_as(w_down))


# ----------------------------------------------------------------------------- norms
def _norm_weight_grad(w, dw_buf_needed: bool):
    mg = main_grad_of(w)
    if mg is not None:
        return mg, True
    return torch.zeros_like(w, dtype=torch.float32), False


class RMSNormFn(torch.autograd.Function):
    """h = bf16(w * rmsnorm(x)), x fp32 [.., D]."""

    @staticmethod
    def forward(ctx, x, w, eps):
        shape = x.shape
        x2d = x.reshape(-1, shape[-1]).contiguous().float()
        M, D = x2d.shape
        h = torch.empty(M, D, device=x.device, dtype=torch.bfloat16)
        rstd = torch.empty(M, device=x.device, dtype=torch.float32)
        C().add_rmsnorm_fwd(x2d, None, w, None, h, rstd, eps)
        ctx.save_for_backward(x2d, rstd, w)
        ctx.shape = shape
        return h.view(shape)

    @staticmethod
    def backward(ctx, gh):
        x2d, rstd, w = ctx.saved_tensors
        M, D = x2d.shape
        gh2d = _bf16(gh.reshape(M, D))
        gx = torch.empty(M, D, device=x2d.device, dtype=torch.float32)
        dw, is_main = _norm_weight_grad(w, True)
        scratch = torch.empty(C().rmsnorm_bwd_scratch_numel(M, D), device=x2d.device, dtype=torch.float32)
        C().rmsnorm_bwd(gh2d, x2d, rstd, w, None, gx, None, dw, True, scratch)
        if is_main:
            notify_grad_ready([w])
        return gx.view(ctx.shape), (None if is_main else dw), None


class AddRMSNormFn(torch.autograd.Function):
    """x_out = x + delta (fp32 residual += bf16 branch output); h = bf16(w * rmsnorm(x_out))."""

    @staticmethod
    def forward(ctx, x, delta, w, eps):
        shape = x.shape
        x2d = x.reshape(-1, shape[-1])
        M, D = x2d.shape
        d2d = _bf16(delta.reshape(M, D))
        x_out = torch.empty(M, D, device=x.device, dtype=torch.float32)
        h = torch.empty(M, D, device=x.device, dtype=torch.bfloat16)
        rstd = torch.empty(M, device=x.device, dtype=torch.float32)
        C().add_rmsnorm_fwd(x2d.contiguous(), d2d, w, x_out, h, rstd, eps)
        ctx.save_for_backward(x_out, rstd, w)
        ctx.shape = shape
        ctx.delta_dtype = delta.dtype
        return x_out.view(shape), h.view(shape)

    @staticmethod
    def backward(ctx, g_xout, gh):
        x_out, rstd, w = ctx.saved_tensors
        M, D = x_out.shape
        dw, is_main = _norm_weight_grad(w, True)
        gx = torch.empty(M, D, device=x_out.device, dtype=torch.float32)
        g_delta = torch.empty(M, D, device=x_out.device, dtype=torch.bfloat16)
        scratch = torch.empty(C().rmsnorm_bwd_scratch_numel(M, D), device=x_out.device, dtype=torch.float32)
        gres = None if g_xout is None else g_xout.reshape(M, D).float().contiguous()
        if gh is None:
            gh = torch.zeros(M, D, device=x_out.device, dtype=torch.bfloat16)
        C().rmsnorm_bwd(_bf16(gh.reshape(M, D)), x_out, rstd, w, gres, gx, g_delta, dw, True, scratch)
        if is_main:
            notify_grad_ready([w])
        gd = g_delta.view(ctx.shape)
        if ctx.delta_dtype != torch.bfloat16:
            gd = gx.view(ctx.shape).to(ctx.delta_dtype)
        return gx.view(ctx.shape), gd, (None if is_main else dw), None


# ----------------------------------------------------------------------------- attention
class RotaryAttentionFn(torch.autograd.Function):
    """RoPE (in place on q|k of the packed qkv buffer) + causal flash attention.

    qkv: [B*T, (Hq + 2*Hkv) * D] bf16 straight from the fused QKV projection.
    Returns o: [B*T, Hq*D] bf16 (c_proj input layout)."""

    @staticmethod
    def forward(ctx, qkv, B, T, Hq, Hkv, D, pos_offset, theta, causal):
        qkv = qkv.contiguous()
        cos, sin = rope_tables(D, theta, T + pos_offset, qkv.device)
        C().rope_inplace(qkv, cos, sin, T, pos_offset, Hq + Hkv, D, False)
        o = torch.empty(B * T, Hq * D, device=qkv.device, dtype=torch.bfloat16)
        lse = torch.empty(B, Hq, T, device=qkv.device, dtype=torch.float32)
        scale = 1.0 / math.sqrt(D)
        C().attn_fwd(qkv, qkv, qkv, 0, Hq * D, (Hq + Hkv) * D, B, T, T, Hq, Hkv, D, o, lse, scale, causal, 0)
        ctx.save_for_backward(qkv, o, lse)
        ctx.cfg = (B, T, Hq, Hkv, D, pos_offset, theta, causal, scale)
        return o

    @staticmethod
    def backward(ctx, do):
        qkv, o, lse = ctx.saved_tensors
        B, T, Hq, Hkv, D, pos_offset, theta, causal, scale = ctx.cfg
        do = _bf16(do)
        dqkv = torch.empty_like(qkv)
        dq_acc = torch.empty(B * T, Hq * D, device=qkv.device, dtype=torch.float32)
        delta = torch.empty(C().attn_bwd_scratch_numel(B, Hq, T), device=qkv.device, dtype=torch.float32)
        C().attn_bwd(qkv, qkv, qkv, o, do, 0, Hq * D, (Hq + Hkv) * D, lse, B, T, Hq, Hkv, D, dqkv, 0, dqkv, Hq * D,
                     dqkv, (Hq + Hkv) * D, dq_acc, delta, scale, causal)
        cos, sin = rope_tables(D, theta, T + pos_offset, qkv.device)
        C().rope_inplace(dqkv, cos, sin, T, pos_offset, Hq + Hkv, D, True)
        return dqkv, None, None, None, None, None, None, None, None


def attention_fwd_only(q, k, v, q_col0, k_col0, v_col0, B, T, Tk, Hq, Hkv, D, causal, causal_offset, out=None,
                       want_lse=False):
    """Forward-only flash attention over token-major buffers (inference / prefill)."""
    o = out if out is not None else torch.empty(B * T, Hq * D, device=q.device, dtype=torch.bfloat16)
    lse = torch.empty(B, Hq, T, device=q.device, dtype=torch.float32) if want_lse else None
    C().attn_fwd(q, k, v, q_col0, k_col0, v_col0, B, T, Tk, Hq, Hkv, D, o, lse, 1.0 / math.sqrt(D), causal,
                 causal_offset)
    return o, lse


# ----------------------------------------------------------------------------- embedding
class EmbeddingFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, idx, weight):
        idx_flat = idx.reshape(-1).contiguous()
        out = torch.empty(idx_flat.numel(), weight.shape[1], device=weight.device, dtype=torch.float32)
        C().embedding_fwd(idx_flat, weight.detach().contiguous(), out)
        ctx.save_for_backward(idx_flat)
        ctx.weight = weight
        return out.view(*idx.shape, weight.shape[1])

    @staticmethod
    def backward(ctx, g):
        (idx_flat,) = ctx.saved_tensors
        w = ctx.weight
        g2d = g.reshape(-1, w.shape[1]).float().contiguous()
        mg = main_grad_of(w)
        if mg is not None:
            C().embedding_bwd(idx_flat, g2d, mg)
            notify_grad_ready([w])
            return None, None
        gw = torch.zeros(w.shape, device=w.device, dtype=torch.float32)
        C().embedding_bwd(idx_flat, g2d, gw)
        return None, gw


# ----------------------------------------------------------------------------- LM head + CE
class LMHeadCrossEntropyFn(torch.autograd.Function):
    """Sum over valid tokens of CE(h @ W^T, targets).

    The CE kernel overwrites the bf16 logits with (softmax - onehot) in place, so
    backward is two GEMMs scaled by the incoming scalar gradient read on device."""

    @staticmethod
    def forward(ctx, h, weight, targets, ignore_index):
        h2d = _bf16(h.reshape(-1, h.shape[-1]))
        w16 = bf16_of(weight)
        logits = gemm_nt(h2d, w16)
        loss_rows = torch.empty(h2d.shape[0], device=h.device, dtype=torch.float32)
        C().cross_entropy_fwd(logits, targets.reshape(-1).contiguous(), loss_rows, None, ignore_index, True)
        ctx.save_for_backward(h2d, logits, w16)
        ctx.weight = weight
        ctx.h_shape = h.shape
        ctx.h_dtype = h.dtype
        return loss_rows.sum()

    @staticmethod
    def backward(ctx, g_loss):
        h2d, grad_logits, w16 = ctx.saved_tensors
        alpha = g_loss.detach().reshape(1).float().contiguous()
        dh = gemm_nn(grad_logits, w16, alpha_t=alpha).view(ctx.h_shape)
        if ctx.h_dtype != torch.bfloat16:
            dh = dh.to(ctx.h_dtype)
        (gw,) = weight_grads([ctx.weight], grad_logits, h2d, alpha_t=alpha)
        return dh, gw, None, None


class ChunkedLMHeadCrossEntropyFn(torch.autograd.Function):
    """Sum over valid tokens of CE(h @ W^T, targets) without a full logits buffer.

    Rows are processed in chunks of ``rows``: the forward computes each chunk's logits
    into one reused [rows, V] bf16 buffer and keeps only the per-row loss; the backward
    recomputes the chunk's logits, the CE kernel turns them into (softmax - onehot) in
    place, and the two GEMMs (scaled by the incoming loss gradient read on the device)
    accumulate dh and dW.  Costs one extra LM-head GEMM per micro-step and saves the
    [tokens, V] logits buffer (1.65 GB at 16 K tokens x 50 K vocab)."""

    @staticmethod
    def forward(ctx, h, weight, targets, ignore_index, rows):
        h2d = _bf16(h.reshape(-1, h.shape[-1]))
        w16 = bf16_of(weight)
        N, V = h2d.shape[0], w16.shape[0]
        t = targets.reshape(-1).contiguous()
        loss_rows = torch.empty(N, device=h.device, dtype=torch.float32)
        buf = torch.empty(min(rows, N), V, device=h.device, dtype=torch.bfloat16)
        for r0 in range(0, N, rows):
            r1 = min(N, r0 + rows)
            lg = buf[:r1 - r0]
            C().gemm(h2d[r0:r1], w16, lg, False, False, False, 1.0, None, 0)
            C().cross_entropy_fwd(lg, t[r0:r1], loss_rows[r0:r1], None, ignore_index, False)
        ctx.save_for_backward(h2d, w16, t)
        ctx.weight, ctx.h_shape, ctx.h_dtype = weight, h.shape, h.dtype
        ctx.ignore_index, ctx.rows = ignore_index, rows
        return loss_rows.sum()

    @staticmethod
    def backward(ctx, g_loss):
        h2d, w16, t = ctx.saved_tensors
        rows = ctx.rows
        N, V = h2d.shape[0], w16.shape[0]
        alpha = g_loss.detach().reshape(1).float().contiguous()
        dh = torch.empty(N, h2d.shape[1], device=h2d.device, dtype=torch.bfloat16)
        buf = torch.empty(min(rows, N), V, device=h2d.device, dtype=torch.bfloat16)
        scratch = torch.empty(min(rows, N), device=h2d.device, dtype=torch.float32)
        gw_total = None
        for r0 in range(0, N, rows):
            r1 = min(N, r0 + rows)
            lg = buf[:r1 - r0]
            C().gemm(h2d[r0:r1], w16, lg, False, False, False, 1.0, None, 0)
            C().cross_entropy_fwd(lg, t[r0:r1], scratch[:r1 - r0], None, ctx.ignore_index, True)
            C().gemm(lg, w16, dh[r0:r1], False, True, False, 1.0, alpha, 0)
            (gw,) = weight_grads([ctx.weight], lg, h2d[r0:r1], alpha_t=alpha)
            if gw is not None:
                gw_total = gw if gw_total is None else gw_total.add_(gw)
        dh = dh.view(ctx.h_shape)
        if ctx.h_dtype != torch.bfloat16:
            dh = dh.to(ctx.h_dtype)
        return dh, gw_total, None, None, None


class LMHeadTokenLogProbFn(torch.autograd.Function):
    """Per-token log-probabilities -CE(h @ W^T, targets) (fp32 [N]).

    Same kernels as :class:`LMHeadCrossEntropyFn`; the upstream gradient is per row
    instead of one scalar, so backward scales row r of the in-place (softmax - onehot)
    buffer by -g[r] before the two GEMMs.  Backward reuses that buffer in place, so it
    can run once per forward."""

    @staticmethod
    def forward(ctx, h, weight, targets, ignore_index):
        h2d = _bf16(h.reshape(-1, h.shape[-1]))
        w16 = bf16_of(weight)
        logits = gemm_nt(h2d, w16)
        nll = torch.empty(h2d.shape[0], device=h.device, dtype=torch.float32)
        C().cross_entropy_fwd(logits, targets.reshape(-1).contiguous(), nll, None, ignore_index, True)
        ctx.save_for_backward(h2d, logits, w16)
        ctx.weight = weight
        ctx.h_shape = h.shape
        ctx.h_dtype = h.dtype
        return nll.neg_()

    @staticmethod
    def backward(ctx, g):
        h2d, grad_logits, w16 = ctx.saved_tensors
        grad_logits.mul_(g.detach().neg().reshape(-1, 1))  # d logp / d logits = -(softmax - onehot)
        dh = gemm_nn(grad_logits, w16).view(ctx.h_shape)
        if ctx.h_dtype != torch.bfloat16:
            dh = dh.to(ctx.h_dtype)
        (gw,) = weight_grads([ctx.weight], grad_logits, h2d)
        return dh, gw, None, None


def lm_logits(h: torch.Tensor, weight: torch.Tensor) -> torch.Tensor:
    """Forward-only logits (bf16) for inference."""
    h2d = _bf16(h.reshape(-1, h.shape[-1]))
    return gemm_nt(h2d, bf16_of(weight)).view(*h.shape[:-1], weight.shape[0])
