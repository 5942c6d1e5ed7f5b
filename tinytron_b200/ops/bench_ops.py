"""Kernel microbenchmarks: ``python -m tinytron_b200.ops.bench_ops <what> [--json]``.

Each measurement is CUDA-event timed on the launching stream, after warm-up,
with L2 flushed (a 256 MiB buffer write) before every timed launch.  Results are
reported against the measured peaks in MEASURED_PEAKS.json when present.
"""
from __future__ import annotations

import argparse
import json
import os
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


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("what", choices=["gemm", "all"])
    ap.add_argument("--json", action="store_true")
    args = ap.parse_args()
    out = {}
    if args.what in ("gemm", "all"):
        out["gemm"] = bench_gemm()
    if args.json:
        print(json.dumps(out))
    else:
        for k, rows in out.items():
            print(f"== {k}")
            for r in rows:
                print("  " + "  ".join(f"{a}={b}" for a, b in r.items()))


if __name__ == "__main__":
    main()
