"""Launchers: preset expansion, autotune log parsing, and a tiny CPU pretraining run
through the command-line entry point."""
import os
import subprocess
import sys

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
