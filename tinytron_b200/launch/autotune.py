"""Throughput auto-tuner (reference: scripts/autotune.sh:5-135).

Runs the pretraining launcher over a grid of SEP sizes x per-rank micro-batch sizes,
parses the per-step log line (``tok/sec: X``), averages the steps after the warm-up,
and writes ``autotune_results.csv`` (``SEP_SIZE,BATCH_SIZE,AVG_TOK_SEC,STATUS``) plus
the best configuration.  A run that prints an out-of-memory error is recorded as OOM,
any other failure (non-zero exit, Python traceback, timeout) as ERROR.  Each run is
started in its own process group and only that group is ever signalled.

    python -m tinytron_b200.launch.autotune --preset 0.25B --nproc 8 --sep-sizes 1 2 4 8 \\
        --batch-sizes 1 2 4 8 16 32 --target-steps 100 --warmup-steps 20 [-- extra pretrain flags]

The reference script's environment variables set the defaults of the same flags
(``SEP_SIZES`` / ``BATCH_SIZES`` as space-separated lists, ``TARGET_STEPS``,
``WARMUP_STEPS``, ``DEBUG=1``; ``MODEL_SIZE`` and ``NUM_GPUS`` as its pretraining launcher
reads them), so ``SEP_SIZES="1 2" bash tinytron_b200/launch/autotune.sh`` works as before;
``RUN_SCRIPT`` has no counterpart (the runs always use this framework's pretraining entry).
"""
from __future__ import annotations

import argparse
import csv
import os
import re
import signal
import socket
import subprocess
import sys
import time

_TOK = re.compile(r"tok/sec:\s*([0-9.]+)")
_OOM = re.compile(r"out of memory|OutOfMemoryError|CUDA_ERROR_OUT_OF_MEMORY", re.IGNORECASE)
_ERR = re.compile(r"Traceback \(most recent call last\)|\bError\b")


def parse_log(lines: list[str], warmup_steps: int) -> tuple[float | None, str]:
    """(mean tok/s over the steps after warm-up, status) from a run's output lines."""
    vals = [float(m.group(1)) for ln in lines for m in [_TOK.search(ln)] if m]
    if any(_OOM.search(ln) for ln in lines):
        return None, "OOM"
    if any(_ERR.search(ln) for ln in lines) and not vals:
        return None, "ERROR"
    vals = vals[warmup_steps:]
    if not vals:
        return None, "NO_DATA"
    return sum(vals) / len(vals), "OK"


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def build_command(args, sep: int, bs: int, log_dir: str) -> list[str]:
    seq = args.seq_len
    steps = args.target_steps + args.warmup_steps
    dp = max(1, args.nproc // sep)
    gbs_tokens = bs * sep * seq * dp // sep  # one micro-step per optimizer step: batch per DP rank x DP size
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={args.nproc}",
           "--master-addr=127.0.0.1", f"--master-port={_free_port()}", "-m", "tinytron_b200.launch.pretrain",
           "--preset", args.preset, "--use_mock_data", "--mock_data_num_samples", str(bs * sep * dp * (steps + 2)),
           "--log_dir", log_dir, "--total_batch_size", str(gbs_tokens * sep), "--batch_size", str(bs * sep),
           "--seq_len", str(seq), "--block_size", str(seq), "--max_steps", str(steps), "--warmup_steps", "1",
           "--sep_size", str(sep), "--debug"]
    return cmd + list(args.extra)


def run_one(cmd: list[str], timeout_s: float, echo: bool) -> list[str]:
    proc = subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True, start_new_session=True)
    lines: list[str] = []
    t0 = time.time()
    try:
        for ln in proc.stdout:
            lines.append(ln)
            if echo:
                sys.stdout.write(ln)
            if _OOM.search(ln) or time.time() - t0 > timeout_s:
                break
    finally:
        if proc.poll() is None:
            try:
                os.killpg(proc.pid, signal.SIGTERM)  # only the run's own process group
                proc.wait(timeout=30)
            except Exception:
                os.killpg(proc.pid, signal.SIGKILL)
    if proc.returncode not in (0, None, -signal.SIGTERM) and not any(_TOK.search(x) for x in lines):
        lines.append(f"Error: exit code {proc.returncode}\n")
    return lines


def _env_ints(name: str, default: list[int]) -> list[int]:
    v = os.environ.get(name, "").split()
    return [int(x) for x in v] if v else default


def build_arg_parser() -> argparse.ArgumentParser:
    env = os.environ.get
    ap = argparse.ArgumentParser("autotune")
    ap.add_argument("--preset", default=env("MODEL_SIZE", "0.25B"))
    ap.add_argument("--nproc", type=int, default=int(env("NUM_GPUS", "8")))
    ap.add_argument("--sep-sizes", type=int, nargs="+", default=_env_ints("SEP_SIZES", [1, 2, 4, 8]))
    ap.add_argument("--batch-sizes", type=int, nargs="+", default=_env_ints("BATCH_SIZES", [1, 2, 4, 8, 16, 32]))
    ap.add_argument("--seq-len", type=int, default=4096)
    ap.add_argument("--target-steps", type=int, default=int(env("TARGET_STEPS", "100")))
    ap.add_argument("--warmup-steps", type=int, default=int(env("WARMUP_STEPS", "20")))
    ap.add_argument("--timeout", type=float, default=1800.0, help="seconds per run")
    ap.add_argument("--results", default="autotune_results.csv")
    ap.add_argument("--log-dir", default="logs/autotune")
    ap.add_argument("--debug", action="store_true", default=env("DEBUG", "0") == "1",
                    help="echo every run's output")
    ap.add_argument("extra", nargs=argparse.REMAINDER, help="after --: extra pretrain flags")
    return ap


def main(argv: list[str] | None = None) -> None:
    args = build_arg_parser().parse_args(argv)
    if args.extra and args.extra[0] == "--":
        args.extra = args.extra[1:]
    best = (0.0, None)
    with open(args.results, "w", newline="") as f:
        w = csv.writer(f)
        w.writerow(["SEP_SIZE", "BATCH_SIZE", "AVG_TOK_SEC", "STATUS"])
        for sep in args.sep_sizes:
            for bs in args.batch_sizes:
                print(f"Testing [ SEP_SIZE={sep} | BATCH_SIZE={bs} ]", flush=True)
                lines = run_one(build_command(args, sep, bs, os.path.join(args.log_dir, f"sep{sep}_bs{bs}")),
                                args.timeout, args.debug)
                tps, status = parse_log(lines, args.warmup_steps)
                w.writerow([sep, bs, f"{tps:.2f}" if tps else "", status])
                f.flush()
                print(f"  -> {status}" + (f" {tps:.2f} tok/s" if tps else ""), flush=True)
                if tps and tps > best[0]:
                    best = (tps, (sep, bs))
                if status == "OOM":
                    break  # larger batches at this SEP size will not fit either
    if best[1] is not None:
        print(f"Best: SEP_SIZE={best[1][0]} BATCH_SIZE={best[1][1]} at {best[0]:.2f} tok/s")


if __name__ == "__main__":
    main()
