"""Collective microbenchmarks on the symmetric heap vs NCCL (one process per GPU).

    python -m torch.distributed.run --nnodes=1 --nproc-per-node N --master-addr 127.0.0.1 \\
        -m tinytron_b200.ops.bench_comm [--json]

Each measurement: warm-up, then CUDA events on the launching stream around ``iters``
back-to-back calls, barrier + synchronize on both sides, max over ranks.  Reported per
call: milliseconds, the bytes each rank moves over NVLink (algorithmic), the resulting
GB/s per GPU and its fraction of the measured 770 GB/s per-direction peer bandwidth.

* ZeRO-1 gradient sync of a dense-1.3B-sized flat buffer (1.166 B fp32 elements):
  tt_comm reduce-scatter + clip + AdamW + all-gather (+ bf16 shadow refresh) vs NCCL
  reduce_scatter_tensor + all_gather_into_tensor (+ the fused AdamW kernel).
* one-shot all-reduce (bf16) at the decode size (32 x 2048) and a bulk size (64 MB).
* equal-split all-to-all (Ulysses exchange) of 64 MB.
* the fused Ulysses head<->sequence exchange of the long-context preset (4096 tokens per
  rank, 16 q / 2 kv heads of 128), both directions, vs the same layout change around NCCL.
* the graph-safe two-kernel all-reduce (device epochs) at the decode size.
"""
from __future__ import annotations

import argparse
import json
import os

import torch
import torch.distributed as dist

NVLINK_GBS = 770.0  # measured peer copy, GB/s per direction per GPU


def _timed(fn, iters: int, warmup: int = 3) -> float:
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    dist.barrier()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(iters):
        fn()
    e.record()
    torch.cuda.synchronize()
    dist.barrier()
    t = torch.tensor([s.elapsed_time(e) / iters], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _row(name, ms, nvlink_bytes, extra=None):
    gbs = nvlink_bytes / (ms / 1e3) / 1e9 if ms > 0 else 0.0
    r = {"op": name, "ms": round(ms, 4), "nvlink_bytes_per_gpu": int(nvlink_bytes), "GBps_per_gpu": round(gbs, 1),
         "frac_of_770GBps": round(gbs / NVLINK_GBS, 3)}
    if extra:
        r.update(extra)
    return r


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--json", action="store_true")
    ap.add_argument("--params", type=int, default=1_166_000_000, help="flat buffer elements (ZeRO-1 case)")
    args = ap.parse_args()
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    W, rank = dist.get_world_size(), dist.get_rank()
    from tinytron_b200.ops import _ext, check_status
    from tinytron_b200.parallel.symm import HeapAllToAll, SymmetricHeap

    C = _ext.load()
    rows = []
    # ---------------------------------------------------------------- ZeRO-1 step
    n = (args.params + 64 * W - 1) // (64 * W) * (64 * W)
    shard = n // W
    lo, hi = rank * shard, (rank + 1) * shard
    heap = SymmetricHeap.create(SymmetricHeap.bytes_needed((n, torch.float32), (n, torch.float32),
                                                           (n, torch.bfloat16)))
    data, grad, p16 = heap.alloc(n, torch.float32), heap.alloc(n, torch.float32), heap.alloc(n, torch.bfloat16)
    data.normal_()
    grad.normal_()
    m, v = torch.zeros(shard, device="cuda"), torch.zeros(shard, device="cuda")
    normc = torch.zeros(2, device="cuda")
    step = {"i": 0}

    def native():
        step["i"] += 1
        heap.reduce_scatter_sumsq(grad, lo, hi, n, 1.0 / W)
        heap.adamw_allgather(data, grad, p16, m, v, lo, hi, 1e-4, (0.9, 0.95), 1e-8, 0.1, step["i"], 1.0,
                             norm_out=normc)
        heap.shadow_refresh(data, p16, lo, hi)

    # bytes over NVLink per GPU: RS reads (W-1)/W of the fp32 buffer, AG writes (W-1)/W of it
    zb = 2 * 4 * n * (W - 1) / W
    rows.append(_row("zero1_step_ttcomm", _timed(native, 3), zb, {"numel": n}))
    heap.close()
    del data, grad, p16
    torch.cuda.empty_cache()
    g = torch.randn(n, device="cuda")
    d = torch.randn(n, device="cuda")
    d16 = torch.empty(n, device="cuda", dtype=torch.bfloat16)
    sq, sc = torch.zeros(2, device="cuda"), torch.empty(4096, device="cuda")
    normt, coef = torch.zeros(1, device="cuda"), torch.ones(1, device="cuda")

    def nccl():
        step["i"] += 1
        dist.reduce_scatter_tensor(g[lo:hi], g, op=dist.ReduceOp.AVG)
        C.sumsq(g[lo:hi], sq[0:1], sc, False)
        dist.all_reduce(sq)
        C.clip_coef(sq[0:1], normt, coef, 1.0)
        C.adamw_step(d[lo:hi], g[lo:hi], m, v, d16[lo:hi], 1e-4, 0.9, 0.95, 1e-8, 0.1, step["i"], coef)
        dist.all_gather_into_tensor(d, d[lo:hi])
        d16.copy_(d)

    rows.append(_row("zero1_step_nccl", _timed(nccl, 3), zb, {"numel": n}))
    del g, d, d16
    torch.cuda.empty_cache()
    # ---------------------------------------------------------------- all-reduce
    for numel, tag in ((32 * 2048, "decode_32x2048"), (32 * 1024 * 1024, "bulk_64MB")):
        h = SymmetricHeap.create(SymmetricHeap.bytes_needed((numel, torch.bfloat16), (numel, torch.bfloat16)))
        slots = [h.alloc(numel, torch.bfloat16), h.alloc(numel, torch.bfloat16)]
        for s in slots:
            s.normal_()
        out = torch.empty(numel, device="cuda", dtype=torch.bfloat16)
        it = {"i": 0}

        def ar():
            it["i"] ^= 1
            h.all_reduce(slots[it["i"]], out)

        x = torch.randn(numel, device="cuda").bfloat16()
        b = 2 * numel * (W - 1)  # one-shot: each rank reads W-1 peer copies
        iters = 200 if numel < 1e6 else 10
        rows.append(_row(f"allreduce_{tag}_ttcomm", _timed(ar, iters), b))
        rows.append(_row(f"allreduce_{tag}_nccl", _timed(lambda: dist.all_reduce(x), iters), b))
        h.close()
    # ---------------------------------------------------------------- all-to-all
    numel = 32 * 1024 * 1024
    a2a = HeapAllToAll(None)
    src = torch.randn(W, numel // W, device="cuda").bfloat16()

    def heap_a2a():
        slot = a2a.slot(src.shape, src.dtype)
        slot.copy_(src)
        a2a.exchange(slot)

    out = torch.empty_like(src)
    b = 2 * numel * (W - 1) / W
    rows.append(_row("alltoall_64MB_ttcomm", _timed(heap_a2a, 10), b))
    rows.append(_row("alltoall_64MB_nccl", _timed(lambda: dist.all_to_all_single(out, src), 10), b))
    # ---------------------------------------------------------------- Ulysses (SEP attention)
    # Long-context preset: one 4096-token chunk per rank, 16 q / 2 kv heads of 128.  Fused:
    # pack + peer-load exchange kernels on a symmetric heap; baseline: the same layout
    # change with torch copies around NCCL all_to_all_single (a separate, unregistered group).
    from tinytron_b200.parallel.symm import enable_heap_all_to_all
    from tinytron_b200.parallel.ulysses import gather_heads_from_ranks, route_heads_to_ranks

    Bu, Tl, Hq, Hkv, D = 1, 4096, 16, 2, 128
    if Hq % W == 0:
        enable_heap_all_to_all(None, torch.device("cuda", local))
        plain = dist.new_group(list(range(W)))
        qkv = torch.randn(Bu * Tl, (Hq + 2 * Hkv) * D, device="cuda").bfloat16()
        full, hq_l, hkv_l = route_heads_to_ranks(qkv, Bu, Tl, Hq, Hkv, D, W, None)
        b_in = full.numel() * 2 * (W - 1) / W  # bytes each rank receives from peers
        rows.append(_row("ulysses_qkv_to_heads_fused", _timed(
            lambda: route_heads_to_ranks(qkv, Bu, Tl, Hq, Hkv, D, W, None), 20), b_in))
        rows.append(_row("ulysses_qkv_to_heads_nccl", _timed(
            lambda: route_heads_to_ranks(qkv, Bu, Tl, Hq, Hkv, D, W, plain), 20), b_in))
        o = torch.randn(Bu * W * Tl, hq_l * D, device="cuda").bfloat16()
        b_out = o.numel() * 2 * (W - 1) / W
        rows.append(_row("ulysses_o_to_tokens_fused", _timed(
            lambda: gather_heads_from_ranks(o, Bu, Tl, Hq, D, W, None), 20), b_out))
        rows.append(_row("ulysses_o_to_tokens_nccl", _timed(
            lambda: gather_heads_from_ranks(o, Bu, Tl, Hq, D, W, plain), 20), b_out))
    # ---------------------------------------------------------------- graph-safe all-reduce
    # decode-sized (32 x 2048 bf16) two-kernel all-reduce with device epochs, as replayed
    # inside the SEP decode graph, against NCCL
    numel = 32 * 2048
    h = SymmetricHeap.create(2 * numel * 2 + 4096)
    slot_buf, slot_bytes = h.replay_slots(numel * 2)
    xin = torch.randn(numel, device="cuda").bfloat16()
    xout = torch.empty_like(xin)

    def replay_ar():
        h.replay_publish(slot_buf, slot_bytes, xin)
        h.replay_reduce(slot_buf, slot_bytes, xout)

    rows.append(_row("allreduce_decode_32x2048_replay", _timed(replay_ar, 200), 2 * numel * (W - 1)))
    h.close()
    check_status()
    if rank == 0:
        if args.json:
            print(json.dumps({"world": W, "rows": rows}))
        else:
            for r in rows:
                print("  ".join(f"{k}={v}" for k, v in r.items()))
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
