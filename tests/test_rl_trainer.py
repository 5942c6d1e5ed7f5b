"""The RL trainer end to end: GRPOTrainer runs optimizer steps (batched rollout through
the inference engine, actor log-probs through the fused LM-head path, GRPO loss, flat
ZeRO-1 AdamW) on CPU as one process and as two gloo ranks (DP=2, and SEP=2), and on
one GPU; plus the per-token log-prob op against an fp32 log-softmax."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from tinytron_b200.training import build_config, parse_args


def _cfg(tmp_path, steps=2, sep=1, world=1, extra=(), hidden=64):
    # seq_len 8 and 9 new tokens: prompt_len + max_new_tokens - 1 = 16 splits over SEP=2
    argv = ["--use_mock_data", "--deterministic", "--mock_data_num_samples", "16", "--log_dir", str(tmp_path),
            "--total_batch_size", str(2 * 8 * 2 * (world // sep)), "--batch_size", "2", "--seq_len", "8",
            "--max_steps", str(steps + 1), "--warmup_steps", "1", "--max_lr", "1e-3", "--min_lr", "1e-4",
            "--num_layer", "2", "--hidden_size", str(hidden), "--num_attention_heads", "4",
            "--num_key_value_heads", "2", "--intermediate_size", "256", "--vocab_size", "128", "--block_size", "64",
            "--init_std", "0.02", "--backend", "gloo", "--sep_size", str(sep), *extra]
    return build_config(parse_args(argv))


def _run_grpo(cfg, steps, device_check=None):
    from tinytron_b200.rl import GRPOTrainer, RLConfig

    tr = GRPOTrainer(cfg, RLConfig(max_new_tokens=9, group_size=2, temperature=1.0, kl_coef=0.0))
    w0 = tr.flat.data.clone()
    results = []
    for s in range(steps):
        tr.one_step_results = {}
        tr._one_training_step(cfg, s)
        results.append({k: (float(v) if torch.is_tensor(v) else v) for k, v in tr.one_step_results.items()})
    moved = (tr.flat.data - w0).abs().max().item()
    tr.close()
    return results, moved


def _clear_env(monkeypatch):
    for k in ("RANK", "WORLD_SIZE", "LOCAL_RANK", "MASTER_ADDR", "MASTER_PORT"):
        monkeypatch.delenv(k, raising=False)


def test_grpo_trainer_two_steps_cpu(tmp_path, monkeypatch):
    _clear_env(monkeypatch)
    res, moved = _run_grpo(_cfg(tmp_path), steps=2)
    assert len(res) == 2
    for r in res:
        for k in ("loss", "reward", "kl", "grad_norm"):
            assert torch.isfinite(torch.tensor(r[k])), (k, r)
        assert r["valid_tokens"] > 0
        assert 0.0 <= r["reward"] <= 1.0
    assert moved > 0.0  # the optimizer updated the actor


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank_entry(rank, world, port, sep, tmp, out):
    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank), MASTER_ADDR="127.0.0.1",
                      MASTER_PORT=str(port))
    torch.set_num_threads(1)
    res, moved = _run_grpo(_cfg(tmp, sep=sep, world=world), steps=2)
    torch.save({"res": res, "moved": moved}, os.path.join(out, f"r{rank}.pt"))


@pytest.mark.parametrize("sep", [1, 2])
def test_grpo_trainer_two_gloo_ranks(tmp_path, sep):
    out = str(tmp_path)
    mp.spawn(_rank_entry, args=(2, _port(), sep, str(tmp_path / "logs"), out), nprocs=2, join=True)
    r0, r1 = torch.load(os.path.join(out, "r0.pt")), torch.load(os.path.join(out, "r1.pt"))
    for a, b in zip(r0["res"], r1["res"]):
        # the step metrics are reduced over the group: every rank reports the same values
        for k in ("loss", "reward", "grad_norm", "valid_tokens"):
            assert abs(a[k] - b[k]) <= 1e-6 * max(1.0, abs(a[k])), (k, a[k], b[k])
    assert r0["moved"] > 0 and r1["moved"] > 0


def test_token_log_probs_cpu_matches_log_softmax():
    from tinytron_b200.models import GPT, ModelConfig

    cfg = ModelConfig(block_size=32, vocab_size=96, num_layer=2, num_attention_heads=4, num_key_value_heads=2,
                      hidden_size=64, intermediate_size=96, init_std=0.02, seed=3)
    m = GPT(cfg, device="cpu")
    g = torch.Generator().manual_seed(0)
    x = torch.randint(0, 96, (2, 16), generator=g)
    y = torch.randint(0, 96, (2, 16), generator=g)
    y[0, :3] = -100
    lp = m.token_log_probs(x, y)
    logits = m(x)
    ref = torch.log_softmax(logits.float(), -1).gather(-1, y.clamp_min(0).unsqueeze(-1)).squeeze(-1)
    ref = ref.masked_fill(y == -100, 0.0)
    assert torch.allclose(lp, ref, atol=1e-5)


@pytest.mark.gpu
def test_lm_head_token_logprobs_gpu_matches_fp32():
    from tinytron_b200 import ops
    from tinytron_b200.ops import _ext, check_status

    _ext.load()
    g = torch.Generator(device="cuda").manual_seed(0)
    N, H, V = 300, 256, 1000
    h = (torch.randn(N, H, device="cuda", generator=g)).bfloat16().requires_grad_(True)
    w = (torch.randn(V, H, device="cuda", generator=g) * 0.05).requires_grad_(True)
    t = torch.randint(0, V, (N,), device="cuda", generator=g)
    t[:7] = -100
    up = torch.randn(N, device="cuda", generator=g)
    lp = ops.lm_head_token_logprobs(h, w, t)
    (lp * up).sum().backward()
    check_status()
    hf, wf = h.detach().float().requires_grad_(True), w.detach().bfloat16().float().requires_grad_(True)
    ref = -torch.nn.functional.cross_entropy(hf @ wf.t(), t, ignore_index=-100, reduction="none")
    (ref * up).sum().backward()
    assert (lp - ref).abs().max().item() < 3e-2
    rel = lambda a, b: ((a.float() - b).norm() / b.norm()).item()  # noqa: E731
    assert rel(h.grad, hf.grad) < 2e-2
    assert rel(w.grad, wf.grad) < 2e-2


@pytest.mark.gpu
def test_grpo_trainer_two_steps_gpu(tmp_path, monkeypatch):
    _clear_env(monkeypatch)
    from tinytron_b200.ops import _ext, check_status

    _ext.load()
    res, moved = _run_grpo(_cfg(tmp_path, extra=["--backend", "nccl"], hidden=256), steps=2)  # head_dim 64
    check_status()
    for r in res:
        for k in ("loss", "reward", "grad_norm"):
            assert torch.isfinite(torch.tensor(r[k])), (k, r)
    assert moved > 0.0
