"""Launchers: preset expansion, autotune log parsing, and a tiny CPU pretraining run
through the command-line entry point."""
import os
import subprocess
import sys

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_expand_preset_puts_preset_flags_first():
    from tinytron_b200.launch._presets import expand_preset

    argv = expand_preset(["--batch_size", "2", "--preset", "0.17B-A0.1B", "--num_layer", "3"])
    assert argv[:2] == ["--num_layer", "12"]
    assert "--use_moe" in argv and argv[argv.index("--num_experts") + 1] == "8"
    assert argv[-4:] == ["--batch_size", "2", "--num_layer", "3"]  # explicit flags come last and win


def test_autotune_parse_log():
    from tinytron_b200.launch.autotune import parse_log

    lines = [f"step {i} | loss: 1.0 | dt: 10ms | tok/sec: {100 + i}.0 | MFU: 1.0%\n" for i in range(5)]
    tps, status = parse_log(lines, warmup_steps=2)
    assert status == "OK" and abs(tps - 103.0) < 1e-9
    assert parse_log(["torch.OutOfMemoryError: CUDA out of memory\n"], 0) == (None, "OOM")
    assert parse_log(["Traceback (most recent call last):\n", "ValueError: x\n"], 0) == (None, "ERROR")


def test_pretrain_entry_point_cpu(tmp_path):
    env = dict(os.environ, PYTHONPATH=ROOT)
    for k in ("RANK", "WORLD_SIZE", "LOCAL_RANK", "MASTER_ADDR", "MASTER_PORT"):
        env.pop(k, None)
    cmd = [sys.executable, "-m", "tinytron_b200.launch.pretrain", "--preset", "b200-tiny-cpu", "--use_mock_data",
           "--mock_data_num_samples", "64", "--log_dir", str(tmp_path), "--total_batch_size", "1024",
           "--batch_size", "2", "--seq_len", "64", "--max_steps", "3", "--warmup_steps", "1", "--debug",
           "--num_layer", "1", "--log_every", "1"]
    out = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stderr[-2000:]
    assert out.stdout.count("tok/sec:") == 3, out.stdout[-2000:]


def test_token_shard_dataset_split_and_resume(tmp_path):
    import numpy as np

    from tinytron_b200.training.streaming import TokenShardDataset, write_token_shards

    toks = np.arange(1000) % 997
    write_token_shards(str(tmp_path), toks, tokens_per_chunk=123)  # samples span shard boundaries
    seq = 16
    full = [s["input_ids"].tolist() for s in TokenShardDataset(str(tmp_path), seq)]
    assert len(full) == (1000 - 1) // seq and full[3] == list(range(48, 64))
    ranks = [[s["input_ids"].tolist() for s in TokenShardDataset(str(tmp_path), seq, r, 2)] for r in range(2)]
    assert ranks[0] == full[0::2] and ranks[1] == full[1::2]  # DP ranks interleave samples
    resumed = [s["labels"].tolist() for s in TokenShardDataset(str(tmp_path), seq, 1, 2, global_skip=10)]
    assert resumed[0] == list(range(11 * seq + 1, 12 * seq + 1))


def test_streaming_trainer_checkpoint_resume_cpu(tmp_path):
    """Train 4 steps with checkpoints, then resume from step 1: the resumed run sees the
    same batches as the uninterrupted one from step 2 on."""
    import numpy as np

    for k in ("RANK", "WORLD_SIZE", "LOCAL_RANK", "MASTER_ADDR", "MASTER_PORT"):
        os.environ.pop(k, None)
    from tinytron_b200.training import build_config, parse_args
    from tinytron_b200.training.streaming import StreamingTrainer, write_token_shards

    data = tmp_path / "shards"
    write_token_shards(str(data), np.random.default_rng(0).integers(0, 256, 40000), tokens_per_chunk=5000)

    def make(log_dir, steps):
        argv = ["--dataset_path", str(data), "--log_dir", str(log_dir), "--total_batch_size", str(2 * 32 * 2),
                "--batch_size", "2", "--seq_len", "32", "--max_steps", str(steps), "--warmup_steps", "1",
                "--num_layer", "1", "--hidden_size", "64", "--num_attention_heads", "4", "--num_key_value_heads", "2",
                "--intermediate_size", "96", "--vocab_size", "256", "--block_size", "32", "--backend", "gloo",
                "--do_save", "--save_every_steps", "1", "--log_every", "100"]
        return StreamingTrainer(build_config(parse_args(argv)))

    seen_a = []
    a = make(tmp_path / "a", 4)
    orig = a._next_train_batch
    a._next_train_batch = lambda: (lambda b: (seen_a.append(b["input_ids"].clone()), b)[1])(orig())
    a.train()
    import shutil

    ck = sorted(p for p in os.listdir(a.log_dir) if p.endswith("_meta.pt"))
    assert ck, os.listdir(a.log_dir)
    for p in os.listdir(a.log_dir):  # keep only the step-1 checkpoint
        if not p.startswith("00001") and p != "log.txt":
            full = os.path.join(a.log_dir, p)
            shutil.rmtree(full) if os.path.isdir(full) else os.remove(full)
    seen_b = []
    b = make(tmp_path / "a", 4)
    orig_b = b._next_train_batch
    b._next_train_batch = lambda: (lambda x: (seen_b.append(x["input_ids"].clone()), x)[1])(orig_b())
    b.train()
    assert b.start_step == 2
    ga = 2
    assert len(seen_b) == 2 * ga
    for x, y in zip(seen_b, seen_a[2 * ga:]):
        assert torch.equal(x, y)


def test_shell_launchers_parse():
    for name in ("pretrain.sh", "inference.sh", "rl.sh", "autotune.sh"):
        out = subprocess.run(["bash", "-n", os.path.join(ROOT, "tinytron_b200", "launch", name)], capture_output=True)
        assert out.returncode == 0, (name, out.stderr)


def _launcher_args(tmp_path, env_extra):
    """Run launch/pretrain.sh with `python` replaced by a stub that prints its arguments."""
    stub = tmp_path / "bin"
    stub.mkdir(exist_ok=True)
    (stub / "python").write_text('#!/bin/bash\nprintf "%s\\n" "$@"\n')
    (stub / "python").chmod(0o755)
    env = {k: v for k, v in os.environ.items() if k not in ("MAX_STEPS", "DO_SAVE", "USE_DISTRIBUTED_OPTIMIZER")}
    env.update(PATH=f"{stub}:{env['PATH']}", LOG_DIR=str(tmp_path / "logs"), **env_extra)
    out = subprocess.run(["bash", os.path.join(ROOT, "tinytron_b200", "launch", "pretrain.sh")], env=env,
                         capture_output=True, text=True, check=True)
    args = out.stdout.split("\n")
    return args[args.index("tinytron_b200.launch.pretrain") + 1:-1]


def test_pretrain_launcher_budget_and_switches(tmp_path):
    """MAX_STEPS replaces the epoch budget (both together are rejected when they
    disagree); DO_SAVE / USE_DISTRIBUTED_OPTIMIZER / LOG_EVERY / SAVE_EVERY_STEPS map to
    their flags; the produced command line parses."""
    from tinytron_b200.launch._presets import expand_preset
    from tinytron_b200.training import parse_args

    a = _launcher_args(tmp_path, {})
    assert "--max_epochs" in a and "--max_steps" not in a and "--do_save" in a and "--use_distributed_optimizer" in a
    b = _launcher_args(tmp_path, {"MAX_STEPS": "10", "DO_SAVE": "0", "USE_DISTRIBUTED_OPTIMIZER": "0",
                                  "LOG_EVERY": "3", "SAVE_EVERY_STEPS": "7"})
    assert b[b.index("--max_steps") + 1] == "10" and "--max_epochs" not in b
    assert "--do_save" not in b and "--use_distributed_optimizer" not in b
    assert b[b.index("--log_every") + 1] == "3" and b[b.index("--save_every_steps") + 1] == "7"
    ns = parse_args(expand_preset(b))
    assert ns.max_steps == 10 and ns.max_epochs is None and not ns.do_save and ns.log_every == 3
    from tinytron_b200.training import build_config

    build_config(ns)  # the static validation (warmup < max_steps, ...) passes
    build_config(parse_args(expand_preset(a)))


def _launcher_module_args(tmp_path, script, module, env_extra):
    stub = tmp_path / "bin"
    stub.mkdir(exist_ok=True)
    (stub / "python").write_text('#!/bin/bash\nprintf "%s\\n" "$@"\n')
    (stub / "python").chmod(0o755)
    env = dict(os.environ)
    env.update(PATH=f"{stub}:{env['PATH']}", LOG_DIR=str(tmp_path / "logs"), **env_extra)
    out = subprocess.run(["bash", os.path.join(ROOT, "tinytron_b200", "launch", script)], env=env,
                         capture_output=True, text=True, check=True)
    args = out.stdout.split("\n")
    return args[args.index(module) + 1:-1]


@pytest.mark.parametrize("sep", ["1", "2"])
def test_inference_and_rl_launchers_produce_parsable_command_lines(tmp_path, sep):
    """The inference and RL shell launchers (single process and torchrun forms) hand their
    entry points command lines that those entry points' parsers accept."""
    from tinytron_b200.inference.arguments import build_parser
    from tinytron_b200.launch._presets import expand_preset
    import argparse

    from tinytron_b200.launch.rl import add_all_arguments, add_rl_args
    from tinytron_b200.training import build_config

    a = _launcher_module_args(tmp_path, "inference.sh", "tinytron_b200.launch.inference",
                              {"SEP_SIZE": sep, "MODEL_SIZE": "0.1B"})
    build_parser().parse_args(expand_preset(a))
    b = _launcher_module_args(tmp_path, "rl.sh", "tinytron_b200.launch.rl", {"SEP_SIZE": sep, "MODEL_SIZE": "0.03B"})
    ns = add_rl_args(add_all_arguments(argparse.ArgumentParser("rl", allow_abbrev=False))).parse_args(expand_preset(b))
    build_config(ns)  # the static validation of the training config passes


def test_autotune_reads_the_reference_environment(monkeypatch):
    """The reference autotune script's variables set the tuner's defaults; flags win."""
    from tinytron_b200.launch.autotune import build_arg_parser

    for k, v in {"SEP_SIZES": "1 2", "BATCH_SIZES": "4 8 16", "TARGET_STEPS": "30", "WARMUP_STEPS": "5",
                 "DEBUG": "1", "MODEL_SIZE": "0.1B", "NUM_GPUS": "2"}.items():
        monkeypatch.setenv(k, v)
    a = build_arg_parser().parse_args([])
    assert (a.sep_sizes, a.batch_sizes, a.target_steps, a.warmup_steps, a.debug, a.preset, a.nproc) == \
        ([1, 2], [4, 8, 16], 30, 5, True, "0.1B", 2)
    b = build_arg_parser().parse_args(["--sep-sizes", "4", "--target-steps", "9"])
    assert b.sep_sizes == [4] and b.target_steps == 9 and b.batch_sizes == [4, 8, 16]
    monkeypatch.delenv("SEP_SIZES")
    monkeypatch.delenv("DEBUG")
    c = build_arg_parser().parse_args([])
    assert c.sep_sizes == [1, 2, 4, 8] and c.debug is False
