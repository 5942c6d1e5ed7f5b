"""Per-kernel device-time breakdown of one training step of the benchmark config.

    python -m tinytron_b200.utils.step_profile [--layers N] [--micro-batch B] [--seq T] [--top K]

Runs warm-up steps, then one profiled step (torch.profiler / CUPTI activity
records, not timed for the benchmark) and prints the kernels sorted by total
device time with counts and shares, plus the framework-vs-other split.
"""
from __future__ import annotations

import argparse
import collections
import os
import sys


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--layers", type=int, default=24)
    ap.add_argument("--micro-batch", type=int, default=4)
    ap.add_argument("--seq", type=int, default=4096)
    ap.add_argument("--grad-accum", type=int, default=4)
    ap.add_argument("--top", type=int, default=40)
    ap.add_argument("--warmup", type=int, default=2)
    ap.add_argument("--moe", action="store_true", help="the MoE benchmark model (16 layers, 64 experts x 1408, top-8)")
    args = ap.parse_args()
    import torch

    from tinytron_b200.training import build_config, parse_args
    from tinytron_b200.training.trainer import Trainer

    for k in ("RANK", "WORLD_SIZE", "LOCAL_RANK", "MASTER_ADDR"):
        os.environ.pop(k, None)
    B, T, GA = args.micro_batch, args.seq, args.grad_accum
    argv = ["--use_mock_data", "--mock_data_num_samples", str(B * GA * 8), "--log_dir", "/tmp/tt_step_profile",
            "--total_batch_size", str(B * T * GA), "--batch_size", str(B), "--seq_len", str(T), "--max_steps", "50",
            "--warmup_steps", "1", "--num_layer", str(args.layers), "--hidden_size", "2048",
            "--num_attention_heads", "16", "--num_key_value_heads", "4", "--intermediate_size", "5504",
            "--vocab_size", "50304", "--block_size", str(T), "--init_std", "0.02"]
    if args.moe:
        argv += ["--use_moe", "--num_experts", "64", "--num_experts_per_tok", "8", "--moe_intermediate_size", "1408"]
    tr = Trainer(build_config(parse_args(argv)))
    g = torch.Generator().manual_seed(0)
    batches = []
    for _ in range(GA):
        d = torch.randint(0, 50304, (B, T + 1), generator=g)
        batches.append({"input_ids": d[:, :T].cuda(), "labels": d[:, 1:].cuda()})
    it = {"i": 0}

    def nxt():
        b = batches[it["i"] % GA]
        it["i"] += 1
        return b

    tr._next_train_batch = nxt
    for s in range(args.warmup):
        tr.train_step(s)
    torch.cuda.synchronize()
    with torch.profiler.profile(activities=[torch.profiler.ProfilerActivity.CUDA]) as prof:
        tr.train_step(args.warmup)
        torch.cuda.synchronize()
    tot = collections.defaultdict(float)
    cnt = collections.Counter()
    for ev in prof.events():
        if ev.device_type == torch.autograd.DeviceType.CUDA:
            name = ev.name
            key = name.replace("(anonymous namespace)::", "").split("(")[0][:110]
            tot[key] += ev.device_time_total if hasattr(ev, "device_time_total") else ev.cuda_time_total
            cnt[key] += 1
    total = sum(tot.values())
    ours = sum(v for k, v in tot.items() if "tt::" in k)
    print(f"total device time {total / 1e3:.2f} ms; framework kernels {ours / 1e3:.2f} ms "
          f"({100 * ours / max(total, 1):.1f}%), other {(total - ours) / 1e3:.2f} ms")
    for k, v in sorted(tot.items(), key=lambda kv: -kv[1])[: args.top]:
        print(f"{v / 1e3:9.3f} ms {100 * v / total:5.1f}%  n={cnt[k]:5d}  {k}")
    sys.stdout.flush()


if __name__ == "__main__":
    main()
