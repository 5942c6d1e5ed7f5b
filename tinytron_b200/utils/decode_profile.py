"""Per-kernel device-time breakdown of decode steps (the 16-layer x 64-expert MoE decode benchmark model).

    python -m tinytron_b200.utils.decode_profile [--layers 16] [--batch 32] [--prompt 1024] [--steps 8] [--dense]

Builds the inference engine (random init), runs a prefill and a few warm-up decode steps,
then profiles ``--steps`` decode steps (torch.profiler / CUPTI activity records, including
the kernels replayed from the captured CUDA graph) and prints kernels by total device time.
"""
from __future__ import annotations

import argparse
import collections

import torch


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--layers", type=int, default=16)
    ap.add_argument("--batch", type=int, default=32)
    ap.add_argument("--prompt", type=int, default=1024)
    ap.add_argument("--steps", type=int, default=8)
    ap.add_argument("--dense", action="store_true", help="dense MLP instead of the 64-expert MoE")
    ap.add_argument("--top", type=int, default=30)
    args = ap.parse_args()
    from tinytron_b200.inference import InferenceEngine
    from tinytron_b200.models.config import ModelConfig

    kw = dict(num_layer=args.layers, hidden_size=2048, num_attention_heads=16, num_key_value_heads=4,
              intermediate_size=5504, vocab_size=50304, block_size=4096, init_std=0.02)
    if not args.dense:
        kw.update(use_moe=True, num_experts=64, num_experts_per_tok=8, moe_intermediate_size=1408)
    eng = InferenceEngine(ModelConfig(**kw), device="cuda", kv_cache_page_size=16)
    prompt = torch.randint(0, 50304, (args.batch, args.prompt), generator=torch.Generator().manual_seed(0))
    eng.generate(prompt, 4, temperature=1.0, top_k=1)
    torch.cuda.synchronize()
    n = args.steps + 4
    with torch.profiler.profile(activities=[torch.profiler.ProfilerActivity.CUDA]) as prof:
        _, st = eng.generate(prompt, n, temperature=1.0, top_k=1, return_stats=True)
        torch.cuda.synchronize()
    tot, cnt = collections.defaultdict(float), collections.Counter()
    for ev in prof.events():
        if ev.device_type == torch.autograd.DeviceType.CUDA:
            key = ev.name.replace("(anonymous namespace)::", "").split("(")[0][:100]
            tot[key] += ev.device_time_total
            cnt[key] += 1
    total = sum(tot.values())
    print(f"prefill + {n} decode steps: device time {total / 1e3:.2f} ms; engine stats: "
          f"prefill {st.get('prefill_ms_device', 0):.2f} ms, decode {st.get('decode_ms_device', 0):.2f} ms "
          f"({st.get('decode_ms_device', 0) / max(n, 1):.3f} ms/step)")
    for k, v in sorted(tot.items(), key=lambda kv: -kv[1])[: args.top]:
        print(f"{v / 1e3:9.3f} ms {100 * v / total:5.1f}%  n={cnt[k]:5d}  {k}")


if __name__ == "__main__":
    main()
