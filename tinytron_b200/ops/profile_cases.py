"""Small fixed workloads for kernel-profiler captures (one process, one GPU).

    python -m tinytron_b200.ops.profile_cases <case>

Each case builds its inputs, runs the kernels it is named for two or three times and
prints ``ok``.  Inputs are larger than the 126 MB L2 where the kernel streams memory,
and every case holds at most a few GB on the device, so a capture of one kernel with a
full metric set ends within a minute or two.

Cases:

* ``zero1``   the ZeRO-1 step kernels (reduce-scatter + sum of squares, clip + AdamW +
              all-gather by peer stores, bf16 shadow refresh) on 2 emulated ranks (two
              symmetric heaps on one GPU, launched rank by rank with waits disabled, so
              no kernel waits on another); 64 M parameters.
* ``ep``      expert-parallel dispatch (peer-store scatter), the grouped expert GEMMs with
              the push-combine epilogue and the local combine, on 2 emulated ranks;
              MoE preset dims (H 2048, 64 experts x 1408, top-8), 4096 tokens per rank.
* ``decode``  one decode step's attention kernels (RoPE + paged KV append, split-KV
              attention, combine) for batch 32, context 1024, page 16, 16q/4kv heads.
* ``attn_bwd_b4``  flash-attention backward at the training shape (B4 T4096 Hq16 Hkv4 d128).
* ``dswiglu`` the down-projection dgrad GEMM with the fused SwiGLU-backward epilogue
              (M 16384, H 2048, I 5504).
* ``moe_decode``  one decode step of the 64-expert MoE (32 tokens, top-8): grouped
              GEMMs that stream every expert's weights.
"""
from __future__ import annotations

import argparse
import math

import torch


def case_zero1(n: int = 64 * 1024 * 1024, W: int = 2):
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
    for step in (1, 2):
        for r, (h, b) in enumerate(zip(heaps, bufs)):
            h.reduce_scatter_sumsq(b["grad"], r * shard, (r + 1) * shard, n, 1.0 / W)
        for r, (h, b) in enumerate(zip(heaps, bufs)):
            h.adamw_allgather(b["data"], b["grad"], b["p16"], b["m"], b["v"], r * shard, (r + 1) * shard, 1e-4,
                              (0.9, 0.95), 1e-8, 0.1, step, 1.0, norm_out=b["norm"])
        for r, (h, b) in enumerate(zip(heaps, bufs)):
            h.shadow_refresh(b["data"], b["p16"], r * shard, (r + 1) * shard)
    torch.cuda.synchronize()
    check_status()
    for h in heaps:
        h.close()


def case_ep(N: int = 4096, W: int = 2, E: int = 64, k: int = 8, H: int = 2048, I: int = 1408):
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
    for _ in range(2):
        counts = [epc.plan_routes(bufs[r], sels[r]) for r in range(W)]
        plans = [epc.plan_finish(bufs[r], sels[r], counts[r]) for r in range(W)]
        xrs = [epc.dispatch(bufs[r], plans[r], xs[r], True) for r in range(W)]
        for r in range(W):
            epc.experts_forward(bufs[r], plans[r], xrs[r], w_gu[r], wd[r], I, True)
        for r in range(W):
            epc.combine(bufs[r], plans[r], ws[r], keep_rows=True, push=True)
    torch.cuda.synchronize()
    check_status()
    for b in bufs:
        b.close()


def case_decode(B: int = 32, ctx: int = 1024, Hq: int = 16, Hkv: int = 4, D: int = 128, page: int = 16):
    from tinytron_b200.inference.cache import LayerPagedKVCache
    from tinytron_b200.ops import check_status

    cache = LayerPagedKVCache(B, Hkv, D, ctx + 16, page, "cuda", torch.bfloat16)
    g = torch.Generator(device="cuda").manual_seed(0)
    W = (Hq + 2 * Hkv) * D
    prompt = torch.randn(B * ctx, W, device="cuda", generator=g).bfloat16()
    cache.append_rope(prompt, B, ctx, Hq, Hkv, D, 10000.0)
    cache.advance(ctx)
    cache.reserve(ctx + 16)
    for _ in range(3):
        qkv = torch.randn(B, W, device="cuda", generator=g).bfloat16()
        q = cache.append_rope(qkv, B, 1, Hq, Hkv, D, 10000.0)
        cache.attend_decode(q.view(B, Hq, D), 1.0 / math.sqrt(D))
        cache.advance(1)
    torch.cuda.synchronize()
    check_status()


def case_attn_bwd_b4(B: int = 4, T: int = 4096, Hq: int = 16, Hkv: int = 4, d: int = 128):
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
    for _ in range(2):
        C.attn_bwd(qkv, qkv, qkv, o, do, 0, Hq * d, (Hq + Hkv) * d, lse, B, T, Hq, Hkv, d, dqkv, 0, dqkv, Hq * d,
                   dqkv, (Hq + Hkv) * d, dq_acc, delta, sc, True)
    torch.cuda.synchronize()


def case_dswiglu(M: int = 16384, H: int = 2048, I: int = 5504):
    """Down-projection dgrad fused with the SwiGLU backward (dense 1.3B MLP, one micro-batch)."""
    from tinytron_b200.ops import _ext, check_status

    C = _ext.load()
    g = torch.Generator(device="cuda").manual_seed(0)
    dy = torch.randn(M, H, device="cuda", generator=g).bfloat16()
    wd = (torch.randn(H, I, device="cuda", generator=g) * 0.02).bfloat16()
    gu = torch.randn(M, 2 * I, device="cuda", generator=g).bfloat16()
    dgu = torch.empty(M, 2 * I, device="cuda", dtype=torch.bfloat16)
    for _ in range(2):
        C.gemm_dswiglu(dy, wd, gu, dgu, 1.0)
    torch.cuda.synchronize()
    check_status()


def case_moe_decode(N: int = 32, E: int = 64, k: int = 8, H: int = 2048, I: int = 1408):
    """One decode step of the MoE experts (32 tokens, top-8 of 64): routing layout, grouped
    SwiGLU gate|up and down GEMMs (weight-streaming bound), weighted combine."""
    from tinytron_b200 import ops
    from tinytron_b200.ops import check_status

    g = torch.Generator(device="cuda").manual_seed(0)
    x = torch.randn(N, H, device="cuda", generator=g).bfloat16()
    wg = (torch.randn(E, I, H, device="cuda", generator=g) * 0.02).bfloat16()
    wu = (torch.randn(E, I, H, device="cuda", generator=g) * 0.02).bfloat16()
    wd = (torch.randn(E, H, I, device="cuda", generator=g) * 0.02).bfloat16()
    with torch.no_grad():
        for _ in range(3):
            sel = torch.topk(torch.randn(N, E, device="cuda", generator=g), k, -1).indices.to(torch.int32)
            w = torch.softmax(torch.randn(N, k, device="cuda", generator=g), -1)
            ops.moe_experts(x, sel, w, wg, wu, wd)
    torch.cuda.synchronize()
    check_status()


CASES = {"zero1": case_zero1, "ep": case_ep, "decode": case_decode, "attn_bwd_b4": case_attn_bwd_b4,
         "dswiglu": case_dswiglu, "moe_decode": case_moe_decode}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("case", choices=sorted(CASES))
    args = ap.parse_args()
    CASES[args.case]()
    print("ok")


if __name__ == "__main__":
    main()
