"""Functional ops used by the model.  Each op has exactly one GPU implementation
(sm_100a kernels from the in-tree extension, via ``functional``) and a CPU
implementation that restates the reference's PyTorch math in fp32 (the CPU oracle
and the CPU training path).  The device of the input selects the implementation;
there is no fallback between them on the GPU.
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F

from .rope import rope_reference


def _cuda_fn():
    from . import functional

    return functional


def check_status(device=None, clear: bool = True) -> int:
    """Read the device status word written by bounded device-side waits; raise on error."""
    from . import _ext

    dev = torch.cuda.current_device() if device is None else torch.device(device).index or 0
    code = int(_ext.load().status_read(dev))
    if code != 0:
        if clear:
            _ext.load().status_clear(dev)
        raise RuntimeError(f"tinytron_b200 device wait timed out (status code {code}) on cuda:{dev}")
    return code


def _cat_w(weights):
    return weights[0] if len(weights) == 1 else torch.cat(list(weights), 0)


def linear(x: torch.Tensor, *weights: torch.Tensor) -> torch.Tensor:
    """y = x @ cat(weights)^T (several weights sharing the input fuse into one GEMM)."""
    if x.is_cuda:
        return _cuda_fn().LinearFn.apply(x, *weights)
    return F.linear(x, _cat_w(weights))


def rmsnorm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    if x.is_cuda:
        return _cuda_fn().RMSNormFn.apply(x, weight, eps)
    dt = x.dtype
    xf = x.to(torch.float32)
    xf = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    return weight * xf.to(dt)


def add_rmsnorm(x: torch.Tensor, delta: torch.Tensor | None, weight: torch.Tensor, eps: float):
    """(x + delta, rmsnorm(x + delta)); with delta None returns (x, rmsnorm(x))."""
    if delta is None:
        return x, rmsnorm(x, weight, eps)
    if x.is_cuda:
        return _cuda_fn().AddRMSNormFn.apply(x, delta, weight, eps)
    x = x + delta
    return x, rmsnorm(x, weight, eps)


def swiglu_mlp(x: torch.Tensor, w_gate: torch.Tensor, w_up: torch.Tensor, w_down: torch.Tensor) -> torch.Tensor:
    if x.is_cuda:
        return _cuda_fn().SwiGLUMLPFn.apply(x, w_gate, w_up, w_down)
    return F.linear(F.silu(F.linear(x, w_gate)) * F.linear(x, w_up), w_down)


def rotary_attention(qkv: torch.Tensor, B: int, T: int, Hq: int, Hkv: int, D: int, pos_offset: int = 0,
                     theta: float = 10000.0, causal: bool = True) -> torch.Tensor:
    """qkv [B*T, (Hq+2Hkv)*D] -> o [B*T, Hq*D]; RoPE positions pos_offset + t."""
    if qkv.is_cuda:
        return _cuda_fn().RotaryAttentionFn.apply(qkv, B, T, Hq, Hkv, D, pos_offset, theta, causal)
    x = qkv.view(B, T, Hq + 2 * Hkv, D).transpose(1, 2)
    q, k, v = x[:, :Hq], x[:, Hq:Hq + Hkv], x[:, Hq + Hkv:]
    pos = torch.arange(pos_offset, pos_offset + T, device=qkv.device).unsqueeze(0)
    q, k = rope_reference(q, k, pos, theta)
    if Hkv != Hq:
        k = k.repeat_interleave(Hq // Hkv, dim=1)
        v = v.repeat_interleave(Hq // Hkv, dim=1)
    o = F.scaled_dot_product_attention(q, k, v, is_causal=causal)
    return o.transpose(1, 2).reshape(B * T, Hq * D)


def moe_topk_softmax(gate_logits: torch.Tensor, k: int):
    """(weights [N, k] fp32, selected experts [N, k]): the k largest router logits per token,
    descending, and the softmax over them (reference mlp.py:240-244)."""
    if gate_logits.is_cuda:
        return _cuda_fn().RouterTopKFn.apply(gate_logits, k)
    topv, sel = torch.topk(gate_logits, k, dim=-1)
    return F.softmax(topv.float(), dim=-1), sel


def moe_experts(x: torch.Tensor, sel: torch.Tensor, weights: torch.Tensor | None, w_gate: torch.Tensor,
                w_up: torch.Tensor, w_down: torch.Tensor) -> torch.Tensor:
    """y[t] = sum_j weights[t, j] * SwiGLU_{sel[t, j]}(x[t])  (weights None: k == 1, unweighted).

    x [N, H]; expert weights [E, I, H], [E, I, H], [E, H, I]; sel holds local expert ids."""
    if x.is_cuda:
        fn = _cuda_fn()
        needs_grad = torch.is_grad_enabled() and any(
            t is not None and t.requires_grad for t in (x, weights, w_gate, w_up, w_down))
        if not needs_grad and x.shape[0] <= fn.SKINNY_MAX_ROWS and fn.skinny_enabled():
            return fn.moe_experts_decode(x, sel, weights, w_gate, w_up, w_down)
        return fn.MoEExpertsFn.apply(x, sel, weights, w_gate, w_up, w_down)
    N, k = sel.shape
    flat = sel.reshape(-1)
    rep = x.repeat_interleave(k, dim=0)
    out = torch.zeros(N * k, x.shape[-1], dtype=torch.float32, device=x.device)
    for e in torch.unique(flat).tolist():
        idx = torch.nonzero(flat == e).squeeze(-1)
        out[idx] = swiglu_mlp(rep[idx], w_gate[e], w_up[e], w_down[e]).float()
    if weights is not None:
        out = out * weights.reshape(-1, 1).float()
    return out.view(N, k, -1).sum(1).to(x.dtype)


def moe_experts_local(x: torch.Tensor, sel: torch.Tensor, weights: torch.Tensor, w_gate: torch.Tensor,
                      w_up: torch.Tensor, w_down: torch.Tensor, e_lo: int) -> torch.Tensor:
    """Inference with experts sharded over ranks: sum over j of weights[t, j] *
    SwiGLU_{sel[t, j]}(x[t]) restricted to the experts [e_lo, e_lo + E_local) held here
    (``sel`` holds global expert ids; the caller all-reduces the partial sums)."""
    if x.is_cuda:
        return _cuda_fn().moe_experts_local(x, sel, weights, w_gate, w_up, w_down, e_lo)[0]
    E = w_gate.shape[0]
    local = sel - e_lo
    mine = (local >= 0) & (local < E)
    y = moe_experts(x, local.clamp(0, E - 1), weights * mine.to(weights.dtype), w_gate, w_up, w_down)
    return y


def moe_experts_local_published(x, sel, weights, w_gate, w_up, w_down, e_lo: int, ar):
    """CUDA inference with experts sharded over an EP group whose graph-safe heap
    all-reduce is ``ar``: (output, reduced).  For a decode-sized batch the combine publishes
    the partial sums into ``ar`` and the output is already the group sum (reduced True);
    otherwise it is this rank's partial sum."""
    return _cuda_fn().moe_experts_local(x, sel, weights, w_gate, w_up, w_down, e_lo, publish=ar)


def linear_row_parallel(x: torch.Tensor, w16: torch.Tensor, ar):
    """CUDA inference: x @ w16^T summed over the SEP group of the heap all-reduce ``ar``,
    with the publish fused into the GEMM's split-sum kernel; None when not applicable."""
    return _cuda_fn().linear_row_parallel(x, w16, ar) if x.is_cuda else None


def embedding(idx: torch.Tensor, weight: torch.Tensor) -> torch.Tensor:
    if weight.is_cuda:
        return _cuda_fn().EmbeddingFn.apply(idx, weight)
    return F.embedding(idx, weight)


def lm_head_ce_sum(h: torch.Tensor, weight: torch.Tensor, targets: torch.Tensor, ignore_index: int = -100,
                   chunk_rows: int = 0):
    """Sum of token cross-entropies over valid targets of logits = h @ weight^T.
    ``chunk_rows`` > 0 (CUDA): no full logits buffer; chunks of rows are recomputed in
    the backward (one extra LM-head GEMM)."""
    if h.is_cuda:
        if chunk_rows > 0:
            return _cuda_fn().ChunkedLMHeadCrossEntropyFn.apply(h, weight, targets, ignore_index, int(chunk_rows))
        return _cuda_fn().LMHeadCrossEntropyFn.apply(h, weight, targets, ignore_index)
    logits = F.linear(h, weight)
    per = F.cross_entropy(logits.view(-1, logits.size(-1)).float(), targets.reshape(-1), ignore_index=ignore_index,
                          reduction="none")
    valid = (targets.reshape(-1) != ignore_index).to(per.dtype)
    return (per * valid).sum()


def lm_head_token_logprobs(h: torch.Tensor, weight: torch.Tensor, targets: torch.Tensor,
                           ignore_index: int = -100) -> torch.Tensor:
    """Per-token log p(target) (fp32 [N]) of logits = h @ weight^T; ignored targets give 0.
    On CUDA the fused LM-head + CE kernel computes it and its buffer carries the backward."""
    if h.is_cuda:
        return _cuda_fn().LMHeadTokenLogProbFn.apply(h, weight, targets, ignore_index)
    logits = F.linear(h.reshape(-1, h.shape[-1]), weight).float()
    return -F.cross_entropy(logits, targets.reshape(-1), ignore_index=ignore_index, reduction="none")


def lm_logits(h: torch.Tensor, weight: torch.Tensor) -> torch.Tensor:
    if h.is_cuda:
        return _cuda_fn().lm_logits(h, weight)
    return F.linear(h, weight)


def attention_scale(head_dim: int) -> float:
    return 1.0 / math.sqrt(head_dim)
