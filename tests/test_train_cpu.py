"""CPU training parity: framework Trainer (fp32 CPU path, flat ZeRO-1 AdamW) vs the
reference model + torch AdamW + reference LR schedule, same weights and batches
(a shortened dense configuration)."""
import math

import pytest
import torch

import ref_oracle
from tinytron_b200.training import build_config, parse_args


def _args(tmp_path, steps=6, extra=()):
    argv = ["--use_mock_data", "--deterministic", "--mock_data_num_samples", "64", "--log_dir", str(tmp_path),
            "--total_batch_size", str(4 * 64), "--batch_size", "4", "--seq_len", "64", "--max_steps", str(steps),
            "--warmup_steps", "2", "--max_lr", "3e-4", "--min_lr", "3e-5", "--weight_decay", "0.1",
            "--num_layer", "2", "--hidden_size", "64", "--num_attention_heads", "4", "--num_key_value_heads", "2",
            "--intermediate_size", "96", "--vocab_size", "256", "--block_size", "64", "--init_std", "0.02",
            "--backend", "gloo", *extra]
    return parse_args(argv)


def test_trainer_runs_and_loss_decreases(tmp_path, monkeypatch):
    for k in ("RANK", "WORLD_SIZE", "LOCAL_RANK", "MASTER_ADDR"):
        monkeypatch.delenv(k, raising=False)
    from tinytron_b200.training.trainer import Trainer

    cfg = build_config(_args(tmp_path, steps=12, extra=["--max_lr", "3e-3", "--mock_data_num_samples", "4"]))
    tr = Trainer(cfg)
    tr.train()
    losses = [tr.results[s]["loss"].item() for s in sorted(tr.results)]
    assert losses[-1] < losses[0] - 0.05, losses


@pytest.mark.skipif(not ref_oracle.available(), reason="reference not installed under baseline/_ref")
def test_trainer_matches_reference_loop(tmp_path, monkeypatch):
    for k in ("RANK", "WORLD_SIZE", "LOCAL_RANK", "MASTER_ADDR"):
        monkeypatch.delenv(k, raising=False)
    from tinytron_b200.training.trainer import Trainer

    steps = 6
    cfg = build_config(_args(tmp_path, steps=steps))
    tr = Trainer(cfg)
    init_sd = {k: v.detach().clone() for k, v in tr.raw_model.state_dict().items()}
    batches = []
    orig = tr._next_train_batch

    def rec():
        b = orig()
        batches.append({k: v.clone() for k, v in b.items()})
        return b

    tr._next_train_batch = rec
    ours = []
    for s in range(steps):
        tr.train_step(s)
        ours.append(tr.one_step_results["loss"].item())

    ref_oracle.ensure_gloo_world1(port=29612)
    with ref_oracle.cpu_reference():
        from tinytron.distributed import parallel_state
        from tinytron.model import GPT as RefGPT
        from tinytron.model.config import ModelConfig as RefCfg
        from tinytron.training.config import ParallelConfig

        parallel_state.initialize_model_parallel(ParallelConfig(sep_size=1))
        rcfg = RefCfg(**{k: v for k, v in cfg.model.__dict__.items() if k in RefCfg.__dataclass_fields__})
        rm = RefGPT(rcfg)
        rm.load_state_dict(init_sd)
        opt = torch.optim.AdamW(rm.parameters(), lr=3e-4, weight_decay=0.1, betas=(0.9, 0.95), eps=1e-8)

        def lr_at(it, max_steps=steps, warm=2, max_lr=3e-4, min_lr=3e-5):
            if it < warm:
                return max_lr * (it + 1) / warm
            r = (it - warm) / (max_steps - warm)
            return min_lr + 0.5 * (1 + math.cos(math.pi * r)) * (max_lr - min_lr)

        ref = []
        for s in range(steps):
            opt.zero_grad()
            b = batches[s]
            _, loss, ll = rm(b["input_ids"], b["labels"])
            loss.backward()
            rm.clip_grad_norm(1.0)
            for g in opt.param_groups:
                g["lr"] = lr_at(s)
            opt.step()
            ref.append(ll.item())
    for a, b in zip(ours, ref):
        assert abs(a - b) < 1e-4 * max(1.0, abs(b)), (ours, ref)


def test_lm_collator_pads_to_sep_multiple_and_shifts():
    from tinytron_b200.training.data import build_lm_collate_fn

    c = build_lm_collate_fn(seq_len=8, sp_world_size=2)
    out = c([{"input_ids": [1, 2, 3, 4, 5]}, {"input_ids": torch.tensor([7, 8, 9]), "labels": torch.tensor([8, 9, 10])}])
    assert out["input_ids"].tolist() == [[1, 2, 3, 4], [7, 8, 9, 0]]
    assert out["labels"].tolist() == [[2, 3, 4, 5], [8, 9, 10, -100]]
    assert int(out["valid_token_count"]) == 7 and int(out["padded_token_count"]) == 8
    with pytest.raises(ValueError):
        build_lm_collate_fn(seq_len=5, sp_world_size=2)([{"input_ids": list(range(10))}])
    import pickle

    pickle.dumps(c)  # DataLoader workers can receive it


@pytest.mark.skipif(not ref_oracle.available(), reason="reference not installed under baseline/_ref")
@pytest.mark.parametrize("deterministic", [True, False])
def test_mock_data_loader_matches_reference(tmp_path, monkeypatch, deterministic):
    """The reference's own _init_dataset (its MockDataset, DistributedSampler and collate)
    and this trainer's loader yield the same batches: the same token stream for the
    same seed, epoch order and shifting.  The vocabulary is 50304, the range the
    reference always draws from (its mock data ignores the model's vocab_size; this
    framework draws below the model's vocab_size, which is the same at 50304)."""
    for k in ("RANK", "WORLD_SIZE", "LOCAL_RANK", "MASTER_ADDR"):
        monkeypatch.delenv(k, raising=False)
    from tinytron_b200.training.trainer import Trainer

    argv = ["--use_mock_data", "--mock_data_num_samples", "24", "--log_dir", str(tmp_path), "--total_batch_size",
            str(4 * 64), "--batch_size", "4", "--seq_len", "64", "--max_steps", "6", "--warmup_steps", "2",
            "--num_layer", "1", "--hidden_size", "64", "--num_attention_heads", "4", "--num_key_value_heads", "2",
            "--intermediate_size", "96", "--vocab_size", "50304", "--block_size", "64", "--seed", "7",
            "--backend", "gloo"] + (["--deterministic"] if deterministic else [])

    def batches(loader, sampler, epoch, n):
        sampler.set_epoch(epoch)
        out = []
        for i, b in enumerate(loader):
            if i == n:
                break
            out.append({k: v.clone() for k, v in b.items()})
        return out

    torch.manual_seed(123)  # the non-deterministic mode draws from the global generator
    tr = Trainer(build_config(parse_args(argv)))
    torch.manual_seed(123)
    ours = batches(tr.train_loader, tr.train_sampler, 0, 6) + batches(tr.train_loader, tr.train_sampler, 1, 2)
    ref_oracle.ensure_gloo_world1(port=29618)
    with ref_oracle.cpu_reference():
        from tinytron.training.arguments import parse_args as ref_parse
        from tinytron.training.config import build_config as ref_build
        from tinytron.training.trainer import Trainer as RefTrainer

        rt = object.__new__(RefTrainer)  # only the data pipeline: no model, no process groups
        rt.dp_world_size, rt.dp_rank, rt.sp_world_size = 1, 0, 1
        rt._init_dataset(ref_build(ref_parse(argv)))
        torch.manual_seed(123)
        ref = batches(rt.train_loader, rt.train_sampler, 0, 6) + batches(rt.train_loader, rt.train_sampler, 1, 2)
    assert len(ours) == len(ref) == 8
    for i, (o, r) in enumerate(zip(ours, ref)):
        assert set(o) >= {"input_ids", "labels"}, i
        for k in ("input_ids", "labels"):
            assert torch.equal(o[k], r[k]), (i, k)


@pytest.mark.skipif(not ref_oracle.available(), reason="reference not installed under baseline/_ref")
@pytest.mark.parametrize("sp", [1, 2, 4])
def test_collate_matches_reference(sp):
    """Variable-length samples (input_ids only, or pre-shifted input_ids/labels; lists or
    tensors; longer than seq_len) collate to the reference's input_ids/labels and valid
    token count, and raise where it raises.  One deliberate difference: the reference
    computes a length rounded up to the SEP size but pads only to the longest sample, so
    its batch can have a length the sequence split cannot divide; here the batch is padded
    to the rounded length (input 0, label -100, which the loss ignores)."""
    from tinytron_b200.training.data import build_lm_collate_fn

    argv = ["--use_mock_data", "--seq_len", "12", "--batch_size", "2", "--total_batch_size", "24",
            "--max_steps", "3", "--warmup_steps", "1", "--sep_size", str(sp)]
    with ref_oracle.cpu_reference():
        from tinytron.training.arguments import parse_args as ref_parse
        from tinytron.training.config import build_config as ref_build
        from tinytron.training.trainer import Trainer as RefTrainer

        rt = object.__new__(RefTrainer)
        rt.sp_world_size = sp
        ref = rt._build_lm_collate_fn(ref_build(ref_parse(argv)))
    ours = build_lm_collate_fn(seq_len=12, sp_world_size=sp)
    g = torch.Generator().manual_seed(sp)
    cases = [
        [{"input_ids": list(range(1, 8))}, {"input_ids": torch.arange(20, 26)}],  # shifted here
        [{"input_ids": torch.arange(5), "labels": torch.arange(1, 6)},
         {"input_ids": torch.arange(9), "labels": torch.arange(1, 10)}],  # already shifted
        [{"input_ids": torch.randint(0, 100, (30,), generator=g)}],  # cut to seq_len
        [{"input_ids": [3, 4]}, {"input_ids": torch.randint(0, 100, (11,), generator=g)}],
    ]
    for i, batch in enumerate(cases):
        try:
            r = ref(batch)
        except ValueError:
            with pytest.raises(ValueError):
                ours(batch)
            continue
        o = ours(batch)
        w = r["input_ids"].shape[1]
        assert o["input_ids"].shape[1] % sp == 0 and o["input_ids"].shape[1] - w < sp, (i, o["input_ids"].shape, w)
        for k, pad in (("input_ids", 0), ("labels", -100)):
            assert torch.equal(o[k][:, :w], r[k]), (i, k, o[k], r[k])
            assert (o[k][:, w:] == pad).all(), (i, k)
        assert int(o["valid_token_count"]) == int(r["valid_token_count"]), i


@pytest.mark.skipif(not ref_oracle.available(), reason="reference not installed under baseline/_ref")
def test_lr_schedule_matches_reference():
    """Warmup, cosine decay and the floor after max_steps: the same learning rate at every
    step as the reference trainer's scheduler."""
    from tinytron_b200.training.trainer import Trainer

    with ref_oracle.cpu_reference():
        from tinytron.training.trainer import Trainer as RefTrainer

        rt = object.__new__(RefTrainer)
    ours = object.__new__(Trainer)
    for max_steps, warm, hi, lo in ((100, 10, 6e-4, 6e-5), (7, 1, 1e-3, 0.0), (50, 49, 3e-4, 3e-5)):
        for it in range(0, max_steps + 5):
            a = ours._lr_scheduler(it, max_steps, warm, hi, lo)
            b = rt._lr_scheduler(it, max_steps, warm, hi, lo)
            assert a == pytest.approx(b, rel=1e-12, abs=0), (max_steps, warm, it, a, b)
