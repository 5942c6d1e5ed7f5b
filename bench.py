"""Headline benchmark: train tokens/s (whole job) + MFU for the dense ~1.3B GPT
(24L, d2048, 16q/4kv heads, SwiGLU 5504, vocab 50304, seq 4096), micro-batch 4
per GPU, grad-accum 4, DDP + ZeRO-1 AdamW, bf16 compute with fp32 masters.

    python bench.py --gpus N --steps K --warmup W [--impl ours|reference]

For N > 1 launch with torch.distributed.run (one rank per GPU, NCCL).  Rank 0
prints one JSON line.  ``value`` is device-timed (CUDA events on the launching
stream, barrier + synchronize on both sides, max over ranks) with inputs already
on the device; ``e2e`` runs the same steps through the public Trainer API with
every step's inputs copied from pinned host memory and the loss read back.
Inputs (weights, activations, 1.6 GB logits) are far larger than the 126 MB L2,
so no explicit L2 flush is needed between steps.
"""
from __future__ import annotations

import argparse
import json
import os
import socket
import statistics
import subprocess
import sys
import tempfile

ROOT = os.path.dirname(os.path.abspath(__file__))

MODEL_FLAGS = ["--num_layer", "24", "--hidden_size", "2048", "--num_attention_heads", "16",
               "--num_key_value_heads", "4", "--intermediate_size", "5504", "--vocab_size", "50304",
               "--block_size", "4096", "--init_std", "0.02"]
MICRO_BATCH, SEQ, GA = 4, 4096, 4
METRIC = "train_tokens_per_sec_per_box"
MODEL_NAME = "dense-1.3B (24L d2048 16q/4kv I5504 V50304)"
PRESET = "b200-dense-1.3b"
SEP = 1

# MoE training config: MoE GPT, SEP = #GPUs + ZeRO-1, 16L d2048 16q/4kv, 64 experts x SwiGLU 1408,
# top-8, aux 0.01, seq 4096, micro-batch 2 sequences per GPU (reference launcher convention
# --batch_size = 2 x SEP: each rank holds 2 x SEP sequences x 4096/SEP tokens = 8192 tokens).
MOE_FLAGS = ["--num_layer", "16", "--hidden_size", "2048", "--num_attention_heads", "16",
             "--num_key_value_heads", "4", "--intermediate_size", "5504", "--vocab_size", "50304",
             "--block_size", "4096", "--init_std", "0.02", "--use_moe", "--num_experts", "64",
             "--num_experts_per_tok", "8", "--moe_intermediate_size", "1408", "--moe_balance_loss_weight", "0.01"]


# Long-context config: dense GPT, Muon + ZeRO-1, SEP = #GPUs, 16L d2048 16q/2kv,
# SwiGLU 5504 (the intermediate size is not fixed by the benchmark; the same value in both arms), seq 32768 = 4096 per rank
# at SEP 8, micro-batch 1 sequence per GPU (--batch_size = 1 x SEP, the launcher convention).
LONGCTX_FLAGS = ["--num_layer", "16", "--hidden_size", "2048", "--num_attention_heads", "16",
                 "--num_key_value_heads", "2", "--intermediate_size", "5504", "--vocab_size", "50304",
                 "--block_size", "32768", "--init_std", "0.02", "--optimizer", "muon"]


def _select_config(name: str, n_gpus: int) -> None:
    global MODEL_FLAGS, MICRO_BATCH, GA, MODEL_NAME, PRESET, SEP, SEQ
    if name == "moe":
        MODEL_FLAGS = MOE_FLAGS
        MICRO_BATCH, GA, SEP = 2 * n_gpus, 4, n_gpus
        MODEL_NAME = "moe-16L (d2048 16q/4kv, 64 experts x 1408 top-8, V50304)"
        PRESET = "b200-moe-16x64"
    elif name == "longctx":
        MODEL_FLAGS = LONGCTX_FLAGS
        MICRO_BATCH, GA, SEP, SEQ = n_gpus, 4, n_gpus, 32768
        MODEL_NAME = "dense-16L long-context (d2048 16q/2kv I5504 V50304, seq 32768), Muon"
        PRESET = "b200-longctx"


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _train_argv(n_gpus: int, steps: int, log_dir: str) -> list[str]:
    dp = n_gpus // SEP
    return ["--use_mock_data", "--deterministic", "--mock_data_num_samples", str(MICRO_BATCH * GA * dp * (steps + 2)),
            "--log_dir", log_dir, "--total_batch_size", str(MICRO_BATCH * SEQ * GA * dp),
            "--batch_size", str(MICRO_BATCH), "--seq_len", str(SEQ), "--max_steps", str(steps + 1),
            "--warmup_steps", "1", "--max_lr", "3e-4", "--min_lr", "3e-5", "--weight_decay", "0.1",
            "--sep_size", str(SEP), "--use_distributed_optimizer", *MODEL_FLAGS]


class ClockSampler:
    """nvidia-smi clock/throttle sampling during the timed region (rank 0, all GPUs)."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, enabled: bool):
        self.enabled = enabled
        self.proc = None
        self.path = None

    def __enter__(self):
        if self.enabled:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            try:
                self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader",
                                              "-lms", "200"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
            except Exception:
                self.proc = None
        return self

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self, n_gpus: int) -> dict:
        out = {"sm_mhz": None, "sm_max_mhz": None, "reasons": []}
        if not self.path or not os.path.exists(self.path):
            return out
        rows = []
        for line in open(self.path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                idx, sm, smax = int(parts[0]), float(parts[1].split()[0]), float(parts[2].split()[0])
            except ValueError:
                continue
            if idx >= n_gpus:
                continue
            rows.append((sm, smax, parts[5:9]))
        if not rows:
            return out
        loaded = [r for r in rows if r[0] > 600] or rows
        out["sm_mhz"] = statistics.median(r[0] for r in loaded)
        out["sm_max_mhz"] = max(r[1] for r in rows)
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = set()
        for r in loaded:
            for name, val in zip(names, r[2]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        out["reasons"] = sorted(reasons)
        out["samples"] = len(loaded)
        return out


def _setup_dist(n_gpus: int):
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world != n_gpus:
        raise SystemExit(f"--gpus {n_gpus} but WORLD_SIZE={world}; launch N>1 with torch.distributed.run")
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    os.environ.setdefault("RANK", "0")
    os.environ.setdefault("LOCAL_RANK", "0")
    os.environ.setdefault("WORLD_SIZE", "1")
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    os.environ.setdefault("MASTER_PORT", str(_free_port()))
    torch.cuda.set_device(local)
    return rank, local, world


def _max_over_ranks(x: float) -> float:
    import torch
    import torch.distributed as dist

    if not dist.is_initialized() or dist.get_world_size() == 1:
        return x
    t = torch.tensor([x], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _timed(step_fn, steps: int, start_step: int) -> float:
    """ms for `steps` calls, CUDA events, barrier + sync on both sides, max over ranks."""
    import torch
    import torch.distributed as dist

    if dist.is_initialized():
        dist.barrier()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for i in range(steps):
        step_fn(start_step + i)
    e.record()
    torch.cuda.synchronize()
    if dist.is_initialized():
        dist.barrier()
    return _max_over_ranks(s.elapsed_time(e))


def _count_launches(step_fn, step: int, own_marker: str) -> tuple[int, int]:
    """(our kernels, all kernels) launched by one step, from the torch profiler (untimed)."""
    import torch

    mode = os.environ.get("TT_BENCH_PROFILE", "0")
    acts = [torch.profiler.ProfilerActivity.CUDA]
    if mode == "2":  # also CPU ops, to name the op that launched each kernel
        acts.append(torch.profiler.ProfilerActivity.CPU)
    with torch.profiler.profile(activities=acts) as prof:
        step_fn(step)
        torch.cuda.synchronize()
    if mode == "2":
        _print_kernel_origins(prof, own_marker)
    ours = total = 0
    spans = []
    for ev in prof.events():
        if ev.device_type == torch.autograd.DeviceType.CUDA:
            total += 1
            if own_marker and own_marker in ev.name:
                ours += 1
            spans.append((ev.time_range.start, ev.time_range.end, ev.name))
    if mode in ("1", "2") and spans:
        _print_kernel_table(spans)
    return ours, total


def _print_kernel_origins(prof, own_marker: str, top: int = 15) -> None:
    """For the kernels not launched by this framework, the outermost profiled op that
    launched them (an autograd node or a top-level aten op), with counts (stderr)."""
    import collections

    per = collections.defaultdict(lambda: [0.0, collections.Counter()])
    for ev in prof.events():
        for k in getattr(ev, "kernels", []) or []:
            if own_marker and own_marker in k.name:
                continue
            root, chain = ev, [ev.name]
            while root.cpu_parent is not None:
                root = root.cpu_parent
                chain.append(root.name)
            origin = next((c for c in chain if c.startswith("autograd::engine::evaluate_function")), chain[-1])
            per[k.name][0] += k.duration / 1e3
            per[k.name][1][f"{origin} <- {chain[0]}"] += 1
    rank = os.environ.get("RANK", "0")
    for name, (ms, origins) in sorted(per.items(), key=lambda kv: -kv[1][0])[:top]:
        print(f"[rank {rank}] origin {ms:8.3f} ms {name[:80]}: {dict(origins.most_common(3))}", file=sys.stderr)


def _print_kernel_table(spans, top: int = 40) -> None:
    """Per-kernel device time of the profiled step (stderr, this rank): total, share,
    launches, and how much of the step's span had no kernel running at all (idle gaps:
    host synchronisation, launch latency)."""
    import collections

    per = collections.defaultdict(lambda: [0.0, 0])
    for a, b, name in spans:
        per[name][0] += (b - a) / 1e3
        per[name][1] += 1
    spans = sorted(spans)
    busy, cur_a, cur_b = 0.0, spans[0][0], spans[0][1]
    for a, b, _ in spans[1:]:  # union of kernel intervals
        if a > cur_b:
            busy += cur_b - cur_a
            cur_a, cur_b = a, b
        else:
            cur_b = max(cur_b, b)
    busy += cur_b - cur_a
    span = spans[-1][1] - spans[0][0]
    tot = sum(v[0] for v in per.values())
    rank = os.environ.get("RANK", "0")
    print(f"[rank {rank}] profiled step: span {span / 1e3:.2f} ms, some kernel running {busy / 1e3:.2f} ms "
          f"({busy / max(span, 1e-9):.3f}), kernel time {tot:.2f} ms", file=sys.stderr)
    for name, (ms, n) in sorted(per.items(), key=lambda kv: -kv[1][0])[:top]:
        print(f"[rank {rank}] {ms:9.3f} ms {ms / tot:6.1%} n={n:6d}  {name[:110]}", file=sys.stderr)


def _make_device_batches(vocab: int, n: int, seed: int):
    import torch

    g = torch.Generator(device="cpu").manual_seed(seed)
    out = []
    for _ in range(n):
        data = torch.randint(0, vocab, (MICRO_BATCH, SEQ + 1), generator=g)
        out.append({"input_ids": data[:, :SEQ].contiguous(), "labels": data[:, 1:].contiguous()})
    return out


def run(args, impl: str):
    import torch
    import torch.distributed as dist

    rank, local, world = _setup_dist(args.gpus)
    log_dir = tempfile.mkdtemp(prefix=f"tt_bench_{impl}_")
    total_steps = args.warmup + 2 * args.steps + 2
    if impl == "reference":
        sys.path.insert(0, os.path.join(ROOT, "baseline", "_ref"))
        try:
            from tinytron.training import Trainer, build_config, parse_args  # the unmodified reference
        except Exception as exc:  # pragma: no cover
            if rank == 0:
                print(json.dumps({"impl": "reference", "unavailable": f"reference import failed: {exc}"}))
            return
        argv = _train_argv(world, total_steps, log_dir) + ["--debug"]
        if not args.ref_eager and args.config in ("dense", "longctx"):
            # measured faster than eager on B200 (68.6K vs 47.3K tok/s, 1 GPU, dense); with MoE the
            # data-dependent expert shapes exceed dynamo's recompile limit and the step fails, so the
            # MoE reference runs eager
            argv.append("--use_compile")
        cfg = build_config(parse_args(argv))
        trainer = Trainer(cfg)
        trainer._init_profiler(cfg)  # sets profiler_record_fn (train() normally does this)
        if args.config == "moe":
            # The reference's grouped_mm path needs moe_intermediate_size == hidden_size; with 1408 != 2048
            # it raises, so its own padded-bmm path is selected (attribute flip, no source edit).
            for m in trainer.raw_model.modules():
                if hasattr(m, "grouped_gemm_supported"):
                    m.grouped_gemm_supported = False
        own_marker = ""
    else:
        sys.path.insert(0, ROOT)
        from tinytron_b200.ops import _ext
        from tinytron_b200.training import build_config, parse_args
        from tinytron_b200.training.trainer import Trainer

        _ext.load()
        cfg = build_config(parse_args(_train_argv(world, total_steps, log_dir) + args.train_args.split()))
        trainer = Trainer(cfg)
        own_marker = "tt::"
    trainer.model.train()
    ga = trainer.training_info["grad_accum_steps"]
    assert ga == GA, ga

    # ---- device-resident inputs (the `value` measurement); SEP peers share their samples
    dp_rank = rank // SEP
    dev_batches = [{k: v.cuda() for k, v in b.items()} for b in _make_device_batches(50304, ga, seed=1234 + dp_rank)]
    state = {"i": 0}

    def next_dev():
        b = dev_batches[state["i"] % ga]
        state["i"] += 1
        return b

    host_batches = [{k: v.pin_memory() for k, v in b.items()}
                    for b in _make_device_batches(50304, ga, seed=99 + dp_rank)]

    def next_host():
        b = host_batches[state["i"] % ga]
        state["i"] += 1
        return b

    def step_fn(step):
        trainer.one_step_results = {}
        trainer._one_training_step(trainer.config, step)

    losses = []

    def e2e_step_fn(step):
        trainer.one_step_results = {}
        trainer._one_training_step(trainer.config, step)
        losses.append(float(trainer.one_step_results["loss"].item()))  # device -> host read of the result

    # With SEP > 1 the reference's _prepare_local_batch (tinytron/training/trainer.py:339-350)
    # slices each rank's sequence chunk out of the batch and relies on its `.to(cuda)` copy to
    # make the chunk contiguous (its loss calls `.view` on the targets), i.e. its stock input
    # is a host batch from the DataLoader; device-resident batches would stay non-contiguous
    # and fail.  So for SEP > 1 the timed reference step is fed pinned host batches (this
    # framework's arm keeps device-resident batches).
    feed = next_host if (SEP > 1 and impl == "reference") else next_dev
    trainer._next_train_batch = feed
    for w in range(args.warmup):
        step_fn(w)
    torch.cuda.synchronize()
    with ClockSampler(rank == 0 and not args.no_clocks) as clk:
        ms = _timed(step_fn, args.steps, args.warmup)
    clocks = clk.summary(world)

    trainer._next_train_batch = next_host
    e2e_ms = _timed(e2e_step_fn, args.steps, args.warmup + args.steps)
    h2d = ga * MICRO_BATCH * SEQ * 8 * 2  # int64 input_ids + labels per rank per step
    d2h = 4

    trainer._next_train_batch = feed
    launches, all_kernels = _count_launches(step_fn, args.warmup + 2 * args.steps, own_marker)

    dp = world // SEP
    tokens_per_step = MICRO_BATCH * SEQ * ga * dp
    value = tokens_per_step / (ms / args.steps / 1e3)
    e2e_value = tokens_per_step / (e2e_ms / args.steps / 1e3)
    sys.path.insert(0, ROOT)
    from tinytron_b200.models.presets import get_preset
    from tinytron_b200.utils.flops import training_flops_per_microstep

    # per rank: MICRO_BATCH sequences x SEQ/SEP tokens, attention over the full SEQ
    flops_step = training_flops_per_microstep(get_preset(PRESET), MICRO_BATCH, SEQ // SEP, sp=SEP) * ga * world
    achieved = flops_step / (ms / args.steps / 1e3)
    peaks = {}
    try:
        peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    except Exception:
        pass
    measured_peak = float(peaks.get("bf16_tflops", 1590.0)) * 1e12
    out = {
        "metric": METRIC,
        "value": round(value, 1),
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms / args.steps, 3),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic uniform random tokens (seeded), random-init weights N(0,0.02)",
        "config": {"model": MODEL_NAME, "global_batch": MICRO_BATCH * GA * dp, "seq_len": SEQ,
                   "micro_batch": MICRO_BATCH, "grad_accum": GA,
                   "parallelism": (f"sep{SEP}+dp{dp}" if SEP > 1 else f"dp{world}") + "+zero1",
                   "optimizer": ("Muon (ZeRO-1)" if "muon" in MODEL_FLAGS else "AdamW (ZeRO-1)"),
                   "l2": "inputs larger than L2 (no flush needed)",
                   "inputs": ("pinned host batches (the reference slices SEP chunks on the host)"
                              if feed is next_host else "device-resident batches")},
        "mfu": round(achieved / (world * 2.25e15), 4),
        "mfu_of_measured_cublas_peak": round(achieved / (world * measured_peak), 4),
        "model_tflops_per_gpu": round(achieved / world / 1e12, 1),
        "e2e": {"value": round(e2e_value, 1), "unit": "tokens/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "ms_per_step": round(e2e_ms / args.steps, 3)},
        "gpu_launches": launches * args.steps,
        "kernels_per_step": {"ours": launches, "all": all_kernels},
        "clocks": clocks,
        "final_loss": losses[-1] if losses else None,
    }
    if impl == "reference":
        out["impl"] = "reference"
        out.pop("gpu_launches")
        out["reference_flags"] = "mock data, deterministic, ZeRO-1, " + (
            "--use_compile" if "--use_compile" in argv else "eager")
    if rank == 0:
        print(json.dumps(out), flush=True)
    if hasattr(trainer, "close"):
        trainer.close()
    elif dist.is_initialized():
        dist.barrier()
        dist.destroy_process_group()


def run_decode(args, impl: str):
    """Decode config: KV-cache inference of the MoE training config's model (random init),
    batch 32 x 1024-token prompts, greedy decode; device-timed prefill and decode."""
    import torch
    import torch.distributed as dist

    rank, local, world = _setup_dist(args.gpus)
    B, P, NEW = 32, 1024, args.decode_steps
    flags = {"num_layer": 16, "hidden_size": 2048, "num_attention_heads": 16, "num_key_value_heads": 4,
             "intermediate_size": 5504, "vocab_size": 50304, "block_size": 4096, "init_std": 0.02, "use_moe": True,
             "num_experts": 64, "num_experts_per_tok": 8, "moe_intermediate_size": 1408}
    if world > 1:
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    if impl == "reference":
        sys.path.insert(0, os.path.join(ROOT, "baseline", "_ref"))
        from tinytron.distributed import parallel_state
        from tinytron.inference import InferenceEngine
        from tinytron.model.config import ModelConfig
        from tinytron.training.config import ParallelConfig
    else:
        sys.path.insert(0, ROOT)
        from tinytron_b200.inference import InferenceEngine
        from tinytron_b200.models.config import ModelConfig
        from tinytron_b200.parallel import parallel_state
        from tinytron_b200.training.config import ParallelConfig
    if world > 1:
        parallel_state.initialize_model_parallel(ParallelConfig(sep_size=world))
    cfg = ModelConfig(**flags)
    kw = dict(model_config=cfg, device=f"cuda:{local}", dtype=torch.bfloat16, use_paged_kv_cache=args.page_size > 0,
              kv_cache_page_size=max(1, args.page_size))
    eng = InferenceEngine(**kw)
    if impl == "reference":
        for m in eng.model.modules():
            if hasattr(m, "grouped_gemm_supported"):
                m.grouped_gemm_supported = False
    g = torch.Generator().manual_seed(0)
    prompt = torch.randint(0, cfg.vocab_size, (B, P), generator=g)
    gen_kw = dict(temperature=1.0, top_k=1, return_stats=True)  # greedy
    eng.generate(prompt, 8, **gen_kw)  # warm-up (allocations, graph capture paths)
    for _ in range(2):
        eng.generate(prompt, 8, **gen_kw)
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    prompt_host = prompt.pin_memory()  # the timed call copies its prompt from pinned host memory
    with ClockSampler(rank == 0 and not args.no_clocks) as clk:
        s.record()
        toks, stats = eng.generate(prompt_host, NEW, **gen_kw)
        toks_host = toks.cpu()  # device -> host read of the result, inside the timed region
        e.record()
        torch.cuda.synchronize()
    d2h = toks_host.numel() * toks_host.element_size()
    total_ms = _max_over_ranks(s.elapsed_time(e))
    dec_ms = _max_over_ranks(stats.get("decode_ms_device", stats["decode_tokens"] / max(
        stats["decode_tokens_per_sec"], 1e-9) * 1e3))
    pre_ms = _max_over_ranks(stats.get("prefill_ms_device", stats["prefill_tokens"] / max(
        stats["prefill_tokens_per_sec"], 1e-9) * 1e3))
    value = B * NEW / (total_ms / 1e3)
    out = {"metric": "decode_tokens_per_sec_per_box", "value": round(B * stats["decode_tokens"] / B / (dec_ms / 1e3), 1),
           "unit": "tokens/s", "n_gpus": world, "steps": NEW, "warmup": 3, "ms_per_step": round(dec_ms / NEW, 3),
           "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
           "data": "synthetic uniform prompts (seeded), random-init weights N(0,0.02)",
           "config": {"model": "moe-16L (d2048 16q/4kv, 64 experts x 1408 top-8)", "batch": B, "prompt_len": P,
                      "decode_steps": NEW, "kv_cache": f"paged page={args.page_size}" if args.page_size > 0 else
                      "contiguous", "parallelism": f"sep{world}" if world > 1 else "1 GPU"},
           "prefill_tokens_per_sec": round(B * P / (pre_ms / 1e3), 1),
           "e2e": {"value": round(value, 1),
                   "unit": "generated tokens/s through InferenceEngine.generate: the prompt copied from pinned host "
                           "memory, prefill, decode and the generated tokens read back to the host (device-timed); "
                           "byte counts are per generate() call",
                   "h2d_bytes_per_step": prompt.numel() * prompt.element_size(), "d2h_bytes_per_step": d2h},
           "clocks": clk.summary(world)}
    if impl == "reference":
        out["impl"] = "reference"
    if rank == 0:
        print(json.dumps(out), flush=True)
    if dist.is_initialized():
        dist.barrier()
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--ref-eager", action="store_true",
                    help="reference arm: run eager instead of --use_compile (compile is the faster of the two)")
    ap.add_argument("--no-clocks", action="store_true")
    ap.add_argument("--config", choices=["dense", "moe", "longctx", "decode"], default="dense",
                    help="dense: 1.3B DP + ZeRO-1 (headline); moe: 16L x 64 experts, SEP = #GPUs + ZeRO-1; "
                         "longctx: Muon, SEP = #GPUs, seq 32768; decode: KV-cache decode of the MoE model")
    ap.add_argument("--train-args", type=str, default="",
                    help="extra trainer flags for this framework's arm (A/B runs, e.g. '--grad_bucket_mb 0')")
    ap.add_argument("--decode-steps", type=int, default=512)
    ap.add_argument("--page-size", type=int, default=16, help="decode: KV page size (0 = contiguous cache)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    try:
        if args.config == "decode":
            run_decode(args, args.impl)
            return
        _select_config(args.config, args.gpus)
        run(args, args.impl)
    except Exception as exc:  # the reference arm reports why it could not produce a number
        if args.impl != "reference":
            raise
        if int(os.environ.get("RANK", "0")) == 0:
            import traceback

            frames = traceback.extract_tb(exc.__traceback__)
            where = f" (raised at {os.path.basename(frames[-1].filename)}:{frames[-1].lineno})" if frames else ""
            msg = f"{type(exc).__name__}: {str(exc).splitlines()[0] if str(exc) else ''}{where}"[:300]
            traceback.print_exc()
            print(json.dumps({"impl": "reference", "config": args.config, "unavailable": msg}), flush=True)
        sys.stdout.flush()
        os._exit(0)


if __name__ == "__main__":
    main()
