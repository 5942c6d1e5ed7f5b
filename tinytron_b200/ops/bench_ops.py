"""Kernel microbenchmarks: ``python -m tinytron_b200.ops.bench_ops <what> [--json]``.

``gemm`` and ``attn`` sweep the training shapes against cuBLAS / torch SDPA; the fixed
kernel cases (``zero1``, ``ep``, ``decode``, ``attn_bwd_b4``, ``dswiglu``, ``moe_decode``,
``muon`` and its cuBLAS/eager baseline ``muon_torch``) time one workload each
(``--iters``/``--warmup``).

Each measurement is CUDA-event timed on the launching stream, after warm-up,
with L2 flushed (a 256 MiB buffer write) before every timed launch.  Results are
reported against the measured peaks in MEASURED_PEAKS.json when present.
"""
from __future__ import annotations

import argparse
import json
import math
from pathlib import Path

import torch

_FLUSH = None


def _flush_l2():
    global _FLUSH
    if _FLUSH is None:
        _FLUSH = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device="cuda")
    _FLUSH.zero_()


def time_fn(fn, iters: int = 20, warmup: int = 5, flush: bool = True) -> float:
    """Median milliseconds of fn() over iters launches (each with a cold L2)."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    times = []
    for _ in range(iters):
        if flush:
            _flush_l2()
        s = torch.cuda.Event(enable_timing=True)
        e = torch.cuda.Event(enable_timing=True)
        s.record()
        fn()
        e.record()
        torch.cuda.synchronize()
        times.append(s.elapsed_time(e))
    times.sort()
    return times[len(times) // 2]


def measured_peaks() -> dict:
    p = Path(__file__).resolve().parents[2] / "MEASURED_PEAKS.json"
    if p.exists():
        return json.loads(p.read_text())
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "fallback": True}


def bench_gemm(shapes=None):
    from tinytron_b200.ops import _ext

    C = _ext.load()
    peak = measured_peaks()["bf16_tflops"]
    M = 16384
    shapes = shapes or [
        ("qkv fwd", M, 3072, 2048, False, False),
        ("c_proj fwd", M, 2048, 2048, False, False),
        ("gate|up fwd", M, 11008, 2048, False, False),
        ("down fwd", M, 2048, 5504, False, False),
        ("lm_head fwd", M, 50304, 2048, False, False),
        ("qkv dgrad", M, 2048, 3072, False, True),
        ("down dgrad", M, 5504, 2048, False, True),
        ("qkv wgrad", 3072, 2048, M, True, True),
        ("gate|up wgrad", 11008, 2048, M, True, True),
        ("down wgrad", 2048, 5504, M, True, True),
    ]
    rows = []
    for name, m, n, k, a_mn, b_mn in shapes:
        A = torch.randn(m, k, device="cuda").bfloat16()
        B = torch.randn(n, k, device="cuda").bfloat16()
        a = A.t().contiguous() if a_mn else A
        b = B.t().contiguous() if b_mn else B
        wgrad = a_mn and b_mn
        c = torch.zeros(m, n, device="cuda", dtype=torch.float32 if wgrad else torch.bfloat16)
        ours = time_fn(lambda: C.gemm(a, b, c, a_mn, b_mn, wgrad, 1.0, None, 0))
        bt = b if b_mn else b.t()
        at = a.t() if a_mn else a
        ref = time_fn(lambda: torch.matmul(at, bt))
        flops = 2.0 * m * n * k
        rows.append(
            dict(
                op=name, M=m, N=n, K=k, ours_ms=round(ours, 4), cublas_ms=round(ref, 4),
                ours_tflops=round(flops / ours / 1e9, 1), cublas_tflops=round(flops / ref / 1e9, 1),
                frac_of_measured_peak=round(flops / ours / 1e9 / peak, 3),
            )
        )
    return rows


def bench_attention(B=4, T=4096, Hq=16, Hkv=4, d=128, iters=10):
    """Causal GQA flash attention fwd/bwd (packed qkv) vs torch SDPA (expanded kv, as the reference)."""
    import math

    import torch.nn.functional as F

    from tinytron_b200.ops import _ext

    C = _ext.load()
    W = (Hq + 2 * Hkv) * d
    qkv = torch.randn(B * T, W, device="cuda").bfloat16()
    o = torch.empty(B * T, Hq * d, device="cuda", dtype=torch.bfloat16)
    lse = torch.empty(B, Hq, T, device="cuda")
    sc = 1 / math.sqrt(d)
    fwd = lambda: C.attn_fwd(qkv, qkv, qkv, 0, Hq * d, (Hq + Hkv) * d, B, T, T, Hq, Hkv, d, o, lse, sc, True, 0)
    t_fwd = time_fn(fwd, iters=iters)
    do = torch.randn_like(o)
    dqkv = torch.empty_like(qkv)
    dq_acc = torch.empty(B * T, Hq * d, device="cuda")
    delta = torch.empty(C.attn_bwd_scratch_numel(B, Hq, T), device="cuda")
    bwd = lambda: C.attn_bwd(qkv, qkv, qkv, o, do, 0, Hq * d, (Hq + Hkv) * d, lse, B, T, Hq, Hkv, d, dqkv, 0, dqkv,
                             Hq * d, dqkv, (Hq + Hkv) * d, dq_acc, delta, sc, True)
    t_bwd = time_fn(bwd, iters=iters)
    x = qkv.view(B, T, Hq + 2 * Hkv, d).transpose(1, 2)
    q = x[:, :Hq].contiguous().requires_grad_(True)
    k = x[:, Hq:Hq + Hkv].repeat_interleave(Hq // Hkv, 1).contiguous().requires_grad_(True)
    v = x[:, Hq + Hkv:].repeat_interleave(Hq // Hkv, 1).contiguous().requires_grad_(True)
    ref_f = lambda: F.scaled_dot_product_attention(q, k, v, is_causal=True)
    t_ref_f = time_fn(lambda: ref_f(), iters=iters)
    out = ref_f()
    g = torch.randn_like(out)
    t_ref_b = time_fn(lambda: torch.autograd.grad(out, (q, k, v), g, retain_graph=True), iters=iters)
    flops = 4.0 * B * Hq * T * T * d / 2
    res = dict(shape=f"B{B} T{T} Hq{Hq} Hkv{Hkv} d{d} causal", fwd_ms=round(t_fwd, 4), bwd_ms=round(t_bwd, 4),
               sdpa_fwd_ms=round(t_ref_f, 4), sdpa_bwd_ms=round(t_ref_b, 4),
               fwd_tflops=round(flops / t_fwd / 1e9, 1), bwd_tflops=round(2.5 * flops / t_bwd / 1e9, 1),
               sdpa_fwd_tflops=round(flops / t_ref_f / 1e9, 1), sdpa_bwd_tflops=round(2.5 * flops / t_ref_b / 1e9, 1))
    return [res]


# ----------------------------------------------------------------------------- fixed kernel cases
# Each builder sets up one workload and returns (run, close): ``run()`` launches the kernels
# of one iteration, ``close()`` checks the device status word and releases buffers.  Inputs
# exceed the 126 MB L2 where the kernel streams memory and every case holds at most a few
# GB, so ``--iters 2 --warmup 1`` also serves as a short case for a profiler capture.


def _case_zero1(n: int = 64 * 1024 * 1024, W: int = 2):
    from tinytron_b200.ops import check_status
    from tinytron_b200.parallel.symm import SymmetricHeap

    n = (n + 64 * W - 1) // (64 * W) * (64 * W)
    shard = n // W
    heaps = SymmetricHeap.create_emulated(SymmetricHeap.bytes_needed((n, torch.float32), (n, torch.float32),
                                                                     (n, torch.bfloat16)), W)
    bufs = []
    for h in heaps:
        data, grad, p16 = h.alloc(n, torch.float32), h.alloc(n, torch.float32), h.alloc(n, torch.bfloat16)
        data.normal_()
        grad.normal_()
        bufs.append(dict(data=data, grad=grad, p16=p16, m=torch.zeros(shard, device="cuda"),
                         v=torch.zeros(shard, device="cuda"), norm=torch.zeros(2, device="cuda")))
    state = {"step": 0}

    def run():
        state["step"] += 1
        for r, (h, b) in enumerate(zip(heaps, bufs)):
            h.reduce_scatter_sumsq(b["grad"], r * shard, (r + 1) * shard, n, 1.0 / W)
        for r, (h, b) in enumerate(zip(heaps, bufs)):
            h.adamw_allgather(b["data"], b["grad"], b["p16"], b["m"], b["v"], r * shard, (r + 1) * shard, 1e-4,
                              (0.9, 0.95), 1e-8, 0.1, state["step"], 1.0, norm_out=b["norm"])
        for r, (h, b) in enumerate(zip(heaps, bufs)):
            h.shadow_refresh(b["data"], b["p16"], r * shard, (r + 1) * shard)

    def close():
        check_status()
        for h in heaps:
            h.close()

    return run, close


def _case_ulysses(B: int = 2, T: int = 4096, Hq: int = 16, Hkv: int = 2, D: int = 128, W: int = 2):
    """Fused Ulysses q|k|v -> heads exchange of the long-context preset on W emulated ranks
    (W heaps on one GPU; every pack is launched before any exchange): per rank a
    [B * T, (Hq + 2 Hkv) * D] chunk in, its heads over the W chunks out."""
    from tinytron_b200.ops import _ext, check_status
    from tinytron_b200.parallel.symm import SymmetricHeap
    from tinytron_b200.parallel.ulysses import kv_heads_for_rank

    C = _ext.load()
    hq_l = Hq // W
    kv0 = [kv_heads_for_rank(r, W, Hq, Hkv)[0] for r in range(W)]
    hkv_l = kv_heads_for_rank(0, W, Hq, Hkv)[1] - kv0[0]
    Wc = (hq_l + 2 * hkv_l) * D
    nbytes = W * B * T * Wc * 2
    heaps = SymmetricHeap.create_emulated(2 * nbytes + 4096, W)
    slots = [h.replay_slots(nbytes) for h in heaps]
    g = torch.Generator(device="cuda").manual_seed(0)
    qkvs = [torch.randn(B * T, (Hq + 2 * Hkv) * D, device="cuda", generator=g).bfloat16() for _ in range(W)]
    fulls = [torch.empty(B * W * T, Wc, device="cuda", dtype=torch.bfloat16) for _ in range(W)]
    b0 = [c * hq_l * D for c in range(W)]
    b1 = [Hq * D + k * D for k in kv0]
    b2 = [(Hq + Hkv) * D + k * D for k in kv0]

    def run():
        for h, (buf, sb), src in zip(heaps, slots, qkvs):
            C.ul_pack(h.gid, h.offset_of(buf), sb, src, B, T, [T, 0, 1], Wc, hq_l * D, (hq_l + hkv_l) * D, b0, b1, b2)
        for h, (buf, sb), out in zip(heaps, slots, fulls):
            C.ul_exchange(h.gid, h.offset_of(buf), sb, out, B, T, [W * T, T, 1], 0, Wc)

    def close():
        check_status()
        for h in heaps:
            h.close()

    return run, close


def _case_ep(N: int = 4096, W: int = 2, E: int = 64, k: int = 8, H: int = 2048, I: int = 1408):
    from tinytron_b200.ops import check_status
    from tinytron_b200.ops.weights import concat_rows
    from tinytron_b200.parallel import ep_comm as epc

    E_l = E // W
    g = torch.Generator(device="cuda").manual_seed(0)
    xs = [torch.randn(N, H, device="cuda", generator=g).bfloat16() for _ in range(W)]
    sels = [torch.topk(torch.randn(N, E, device="cuda", generator=g), k, -1).indices.to(torch.int32)
            for _ in range(W)]
    ws = [torch.softmax(torch.randn(N, k, device="cuda", generator=g), -1).reshape(-1).contiguous()
          for _ in range(W)]
    w_gu = [concat_rows([(torch.randn(E_l * I, H, device="cuda", generator=g) * 0.02).bfloat16(),
                         (torch.randn(E_l * I, H, device="cuda", generator=g) * 0.02).bfloat16()]) for _ in range(W)]
    wd = [(torch.randn(E_l * H, I, device="cuda", generator=g) * 0.02).bfloat16() for _ in range(W)]
    bufs = epc.EPBuffers.create_emulated(W, E, H, epc.capacity(W, N, k, E_l))

    def run():
        counts = [epc.plan_routes(bufs[r], sels[r]) for r in range(W)]
        plans = [epc.plan_finish(bufs[r], sels[r], counts[r]) for r in range(W)]
        xrs = [epc.dispatch(bufs[r], plans[r], xs[r], True) for r in range(W)]
        for r in range(W):
            epc.experts_forward(bufs[r], plans[r], xrs[r], w_gu[r], wd[r], I, True)
        for r in range(W):
            epc.combine(bufs[r], plans[r], ws[r], keep_rows=True, push=True)

    def close():
        check_status()
        for b in bufs:
            b.close()

    return run, close


def _case_decode(B: int = 32, ctx: int = 1024, Hq: int = 16, Hkv: int = 4, D: int = 128, page: int = 16):
    from tinytron_b200.inference.cache import LayerPagedKVCache
    from tinytron_b200.ops import check_status

    cache = LayerPagedKVCache(B, Hkv, D, ctx + 16, page, "cuda", torch.bfloat16)
    g = torch.Generator(device="cuda").manual_seed(0)
    W = (Hq + 2 * Hkv) * D
    prompt = torch.randn(B * ctx, W, device="cuda", generator=g).bfloat16()
    cache.append_rope(prompt, B, ctx, Hq, Hkv, D, 10000.0)
    cache.advance(ctx)
    cache.reserve(ctx + 16)
    qkv = torch.randn(B, W, device="cuda", generator=g).bfloat16()

    def run():  # one decode step's attention; the cache length is not advanced, so every
        # iteration appends at (and attends over) the same position
        q = cache.append_rope(qkv, B, 1, Hq, Hkv, D, 10000.0)
        cache.attend_decode(q.view(B, Hq, D), 1.0 / math.sqrt(D))

    return run, check_status


def _case_attn_bwd_b4(B: int = 4, T: int = 4096, Hq: int = 16, Hkv: int = 4, d: int = 128):
    from tinytron_b200.ops import _ext

    C = _ext.load()
    W = (Hq + 2 * Hkv) * d
    qkv = torch.randn(B * T, W, device="cuda").bfloat16()
    o = torch.empty(B * T, Hq * d, device="cuda", dtype=torch.bfloat16)
    lse = torch.empty(B, Hq, T, device="cuda")
    sc = 1 / math.sqrt(d)
    C.attn_fwd(qkv, qkv, qkv, 0, Hq * d, (Hq + Hkv) * d, B, T, T, Hq, Hkv, d, o, lse, sc, True, 0)
    do = torch.randn_like(o)
    dqkv = torch.empty_like(qkv)
    dq_acc = torch.empty(B * T, Hq * d, device="cuda")
    delta = torch.empty(C.attn_bwd_scratch_numel(B, Hq, T), device="cuda")

    def run():
        C.attn_bwd(qkv, qkv, qkv, o, do, 0, Hq * d, (Hq + Hkv) * d, lse, B, T, Hq, Hkv, d, dqkv, 0, dqkv, Hq * d,
                   dqkv, (Hq + Hkv) * d, dq_acc, delta, sc, True)

    return run, (lambda: None)


def _case_dswiglu(M: int = 16384, H: int = 2048, I: int = 5504):
    """Down-projection dgrad fused with the SwiGLU backward (dense 1.3B MLP, one micro-batch)."""
    from tinytron_b200.ops import _ext, check_status

    C = _ext.load()
    g = torch.Generator(device="cuda").manual_seed(0)
    dy = torch.randn(M, H, device="cuda", generator=g).bfloat16()
    wd = (torch.randn(H, I, device="cuda", generator=g) * 0.02).bfloat16()
    gu = torch.randn(M, 2 * I, device="cuda", generator=g).bfloat16()
    dgu = torch.empty(M, 2 * I, device="cuda", dtype=torch.bfloat16)
    return (lambda: C.gemm_dswiglu(dy, wd, gu, dgu, 1.0)), check_status


def _case_moe_decode(N: int = 32, E: int = 64, k: int = 8, H: int = 2048, I: int = 1408):
    """One decode step of the MoE experts (32 tokens, top-8 of 64): routing layout, grouped
    SwiGLU gate|up and down GEMMs (weight-streaming bound), weighted combine."""
    from tinytron_b200 import ops
    from tinytron_b200.ops import check_status

    g = torch.Generator(device="cuda").manual_seed(0)
    x = torch.randn(N, H, device="cuda", generator=g).bfloat16()
    wg = (torch.randn(E, I, H, device="cuda", generator=g) * 0.02).bfloat16()
    wu = (torch.randn(E, I, H, device="cuda", generator=g) * 0.02).bfloat16()
    wd = (torch.randn(E, H, I, device="cuda", generator=g) * 0.02).bfloat16()
    sel = torch.topk(torch.randn(N, E, device="cuda", generator=g), k, -1).indices.to(torch.int32)
    w = torch.softmax(torch.randn(N, k, device="cuda", generator=g), -1)

    def run():
        with torch.no_grad():
            ops.moe_experts(x, sel, w, wg, wu, wd)

    return run, check_status


def _case_moe_decode_ep8(N: int = 32, E: int = 64, k: int = 8, H: int = 2048, I: int = 1408, ranks: int = 8):
    """The same decode step for one rank of an EP=8 group: its 8 local experts' share of
    the 32 tokens' pairs (the others go to the never-computed remote segment)."""
    from tinytron_b200 import ops
    from tinytron_b200.ops import check_status

    E_l = E // ranks
    g = torch.Generator(device="cuda").manual_seed(0)
    x = torch.randn(N, H, device="cuda", generator=g).bfloat16()
    wg = (torch.randn(E_l, I, H, device="cuda", generator=g) * 0.02).bfloat16()
    wu = (torch.randn(E_l, I, H, device="cuda", generator=g) * 0.02).bfloat16()
    wd = (torch.randn(E_l, H, I, device="cuda", generator=g) * 0.02).bfloat16()
    sel = torch.topk(torch.randn(N, E, device="cuda", generator=g), k, -1).indices.to(torch.int32)
    w = torch.softmax(torch.randn(N, k, device="cuda", generator=g), -1)

    def run():
        with torch.no_grad():
            ops.moe_experts_local(x, sel, w, wg, wu, wd, 0)

    return run, check_status


def _case_muon(layers: int = 16, H: int = 2048, kv: int = 256, I: int = 5504):
    """One Muon step over the matrices of the long-context preset (16 layers, d2048,
    2 kv heads, SwiGLU 5504) on one GPU: momentum, tcgen05 Newton-Schulz (symmetric
    tiles, fused axpby epilogues, side streams for the k/v matrices), update."""
    from tinytron_b200.optim import Muon

    shapes = [(H, H), (kv, H), (kv, H), (H, H), (I, H), (I, H), (H, I)] * layers
    g = torch.Generator(device="cuda").manual_seed(0)
    params = [torch.nn.Parameter(torch.randn(s, device="cuda", generator=g) * 0.02) for s in shapes]
    for p in params:
        p.grad = torch.randn(p.shape, device="cuda", generator=g)
    opt = Muon([{"params": params, "use_muon": True, "lr": 0.02, "momentum": 0.95, "weight_decay": 0.1}])
    return (lambda: opt.step()), (lambda: None)


def _case_muon_torch(layers: int = 16, H: int = 2048, kv: int = 256, I: int = 5504):
    """The same Muon step written with torch bf16 matmuls (cuBLAS) and eager elementwise
    ops, one matrix after another: the library baseline for ``muon``."""
    a, b, c = 3.4445, -4.7750, 2.0315
    shapes = [(H, H), (kv, H), (kv, H), (H, H), (I, H), (I, H), (H, I)] * layers
    g = torch.Generator(device="cuda").manual_seed(0)
    params = [torch.randn(s, device="cuda", generator=g) * 0.02 for s in shapes]
    grads = [torch.randn(s, device="cuda", generator=g) for s in shapes]
    moms = [torch.zeros(s, device="cuda") for s in shapes]

    def run():
        for p, gr, m in zip(params, grads, moms):
            m.lerp_(gr, 0.05)
            u = gr.lerp(m, 0.95)
            X = u.bfloat16()
            tall = X.size(0) > X.size(1)
            if tall:
                X = X.mT
            X = X / (X.norm() + 1e-7)
            for _ in range(5):
                A = X @ X.mT
                X = a * X + (b * A + c * A @ A) @ X
            if tall:
                X = X.mT
            p.mul_(1 - 0.02 * 0.1).add_(X.float(), alpha=-0.02 * max(1.0, p.size(0) / p.size(1)) ** 0.5)

    return run, (lambda: None)


def _case_norm(M: int = 16384, D: int = 2048):
    """Fused residual-add + RMSNorm forward and backward of one dense-1.3B micro-batch
    (M tokens, fp32 residual stream); 670 MB of algorithmic traffic per iteration."""
    from tinytron_b200.ops import _ext, check_status

    C = _ext.load()
    g = torch.Generator(device="cuda").manual_seed(0)
    x = torch.randn(M, D, device="cuda", generator=g)
    delta = torch.randn(M, D, device="cuda", generator=g).bfloat16()
    w = torch.rand(D, device="cuda", generator=g) + 0.5
    x_out = torch.empty_like(x)
    h = torch.empty(M, D, device="cuda", dtype=torch.bfloat16)
    rstd = torch.empty(M, device="cuda")
    gh = torch.randn(M, D, device="cuda", generator=g).bfloat16()
    gres = torch.randn(M, D, device="cuda", generator=g)
    gx = torch.empty_like(x)
    gd = torch.empty(M, D, device="cuda", dtype=torch.bfloat16)
    dw = torch.zeros(D, device="cuda")
    scratch = torch.empty(C.rmsnorm_bwd_scratch_numel(M, D), device="cuda")

    def run():
        C.add_rmsnorm_fwd(x, delta, w, x_out, h, rstd, 1e-5)
        C.rmsnorm_bwd(gh, x_out, rstd, w, gres, gx, gd, dw, True, scratch)

    return run, check_status


def _case_ce(M: int = 4096, V: int = 50304):
    """Fused cross-entropy over bf16 logits with the in-place (softmax - onehot) gradient
    (one dense-1.3B micro-batch quarter: 412 MB read + written)."""
    from tinytron_b200.ops import _ext, check_status

    C = _ext.load()
    g = torch.Generator(device="cuda").manual_seed(0)
    logits = torch.randn(M, V, device="cuda", generator=g).bfloat16()
    t = torch.randint(0, V, (M,), device="cuda", generator=g)
    loss = torch.empty(M, device="cuda")
    return (lambda: C.cross_entropy_fwd(logits, t, loss, None, -100, True)), check_status


def _case_router(N: int = 8192, E: int = 64, k: int = 8, H: int = 2048):
    """MoE routing of one SEP=8 micro-batch per rank: router top-k + softmax, expert
    layout (segments, slots), row gather for the grouped GEMMs."""
    from tinytron_b200.ops import _ext, check_status
    from tinytron_b200.ops.functional import moe_align

    C = _ext.load()
    g = torch.Generator(device="cuda").manual_seed(0)
    logits = torch.randn(N, E, device="cuda", generator=g).bfloat16()
    x = torch.randn(N, H, device="cuda", generator=g).bfloat16()
    w = torch.empty(N, k, device="cuda")
    sel = torch.empty(N, k, device="cuda", dtype=torch.int32)
    P = N * k
    align = moe_align(P, E)
    cap = C.moe_row_capacity(P, E, align)
    grp = torch.empty(E + 1, device="cuda", dtype=torch.int32)
    slot = torch.empty(P, device="cuda", dtype=torch.int32)
    row_pair = torch.empty(cap, device="cuda", dtype=torch.int32)
    xr = torch.empty(cap, H, device="cuda", dtype=torch.bfloat16)

    def run():
        C.moe_topk_softmax(logits, k, w, sel)
        C.moe_layout(sel.view(-1), E, grp, slot, row_pair, align)
        C.moe_gather_rows(x, row_pair, grp, k, xr)

    return run, check_status


def _case_sample(B: int = 32, V: int = 50304):
    """One decode step's sampling: temperature, top-k 50, top-p 0.9, Philox draw, log-prob."""
    from tinytron_b200.ops import _ext, check_status

    C = _ext.load()
    g = torch.Generator(device="cuda").manual_seed(0)
    logits = (torch.randn(B, V, device="cuda", generator=g) * 3).bfloat16()
    tok = torch.empty(B, device="cuda", dtype=torch.long)
    lp = torch.empty(B, device="cuda")
    return (lambda: C.sample_tokens(logits, 0.8, 50, 0.9, 1234, 0, tok, lp)), check_status


KERNEL_CASES = {"zero1": _case_zero1, "ep": _case_ep, "decode": _case_decode, "attn_bwd_b4": _case_attn_bwd_b4,
                "dswiglu": _case_dswiglu, "moe_decode": _case_moe_decode, "moe_decode_ep8": _case_moe_decode_ep8, "muon": _case_muon,
                "muon_torch": _case_muon_torch, "norm": _case_norm,
                "muon_2layers": lambda: _case_muon(layers=2), "ce": _case_ce, "router": _case_router,
                "sample": _case_sample, "ulysses": _case_ulysses}


def bench_case(name: str, iters: int, warmup: int) -> list[dict]:
    """Median device ms of one iteration of a fixed kernel case (L2 flushed before each)."""
    run, close = KERNEL_CASES[name]()
    try:
        ms = time_fn(run, iters=iters, warmup=warmup)
    finally:
        torch.cuda.synchronize()
        close()
    return [dict(case=name, ms=round(ms, 4), iters=iters)]


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("what", choices=["gemm", "attn", "attn_fwd_once", "attn_bwd_once", "gemm_once", "all",
                                     *sorted(KERNEL_CASES)])
    ap.add_argument("--json", action="store_true")
    ap.add_argument("--iters", type=int, default=20, help="fixed kernel cases: timed iterations")
    ap.add_argument("--warmup", type=int, default=3, help="fixed kernel cases: untimed iterations")
    args = ap.parse_args()
    out = {}
    if args.what in KERNEL_CASES:
        out[args.what] = bench_case(args.what, args.iters, args.warmup)
    if args.what == "gemm_once":  # small fixed case for profiler captures: gate|up forward GEMM, 2 launches
        from tinytron_b200.ops import _ext

        C = _ext.load()
        M, N, K = 16384, 11008, 2048
        a = torch.randn(M, K, device="cuda").bfloat16()
        b = torch.randn(N, K, device="cuda").bfloat16()
        c = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
        for _ in range(2):
            C.gemm(a, b, c, False, False, False, 1.0, None, 0)
        torch.cuda.synchronize()
        print("ok")
        return
    if args.what == "attn_fwd_once":  # small fixed case for profiler captures
        import math

        from tinytron_b200.ops import _ext

        C = _ext.load()
        B, T, Hq, Hkv, d = 1, 4096, 16, 4, 128
        qkv = torch.randn(B * T, (Hq + 2 * Hkv) * d, device="cuda").bfloat16()
        o = torch.empty(B * T, Hq * d, device="cuda", dtype=torch.bfloat16)
        lse = torch.empty(B, Hq, T, device="cuda")
        for _ in range(2):
            C.attn_fwd(qkv, qkv, qkv, 0, Hq * d, (Hq + Hkv) * d, B, T, T, Hq, Hkv, d, o, lse, 1 / math.sqrt(d), True, 0)
        torch.cuda.synchronize()
        print("ok")
        return
    if args.what == "attn_bwd_once":  # small fixed case for profiler captures: 1 fwd + 2 bwd launches
        import math

        from tinytron_b200.ops import _ext

        C = _ext.load()
        B, T, Hq, Hkv, d = 1, 4096, 16, 4, 128
        W = (Hq + 2 * Hkv) * d
        qkv = torch.randn(B * T, W, device="cuda").bfloat16()
        o = torch.empty(B * T, Hq * d, device="cuda", dtype=torch.bfloat16)
        lse = torch.empty(B, Hq, T, device="cuda")
        sc = 1 / math.sqrt(d)
        C.attn_fwd(qkv, qkv, qkv, 0, Hq * d, (Hq + Hkv) * d, B, T, T, Hq, Hkv, d, o, lse, sc, True, 0)
        do = torch.randn_like(o)
        dqkv = torch.empty_like(qkv)
        dq_acc = torch.empty(B * T, Hq * d, device="cuda")
        delta = torch.empty(C.attn_bwd_scratch_numel(B, Hq, T), device="cuda")
        for _ in range(2):
            C.attn_bwd(qkv, qkv, qkv, o, do, 0, Hq * d, (Hq + Hkv) * d, lse, B, T, Hq, Hkv, d, dqkv, 0, dqkv, Hq * d,
                       dqkv, (Hq + Hkv) * d, dq_acc, delta, sc, True)
        torch.cuda.synchronize()
        print("ok")
        return
    if args.what in ("gemm", "all"):
        out["gemm"] = bench_gemm()
    if args.what in ("attn", "all"):
        out["attn"] = bench_attention()
    if args.json:
        print(json.dumps(out))
    else:
        for k, rows in out.items():
            print(f"== {k}")
            for r in rows:
                print("  " + "  ".join(f"{a}={b}" for a, b in r.items()))


if __name__ == "__main__":
    main()
