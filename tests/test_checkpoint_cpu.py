"""Checkpoint save -> resume round trip through the Trainer, and interoperability of the
checkpoint files with the unmodified reference's loader (CPU)."""
import os

import pytest
import torch

import ref_oracle
from tinytron_b200.training import build_config, parse_args


def _args(log_dir, steps, extra=()):
    argv = ["--use_mock_data", "--deterministic", "--mock_data_num_samples", "64", "--log_dir", str(log_dir),
            "--total_batch_size", str(2 * 64), "--batch_size", "2", "--seq_len", "64", "--max_steps", str(steps),
            "--warmup_steps", "1", "--max_lr", "1e-3", "--min_lr", "1e-4", "--weight_decay", "0.1",
            "--num_layer", "2", "--hidden_size", "64", "--num_attention_heads", "4", "--num_key_value_heads", "2",
            "--intermediate_size", "96", "--vocab_size", "256", "--block_size", "64", "--init_std", "0.02",
            "--do_save", "--save_every_steps", "1000", *extra]
    return build_config(parse_args(argv))


@pytest.fixture
def no_dist_env(monkeypatch):
    for k in ("RANK", "WORLD_SIZE", "LOCAL_RANK", "MASTER_ADDR", "MASTER_PORT"):
        monkeypatch.delenv(k, raising=False)


def test_save_resume_round_trip(tmp_path, no_dist_env):
    """Steps 0..3 in one run == steps 0..2, save, a fresh Trainer resumed from the files,
    step 3 (model, optimizer state, sampler position and RNG restored)."""
    from tinytron_b200.training.trainer import Trainer

    a = Trainer(_args(tmp_path / "a", 6))
    losses_a = [a.train_step(s)["loss"].item() for s in range(4)]
    b = Trainer(_args(tmp_path / "b", 6))
    for s in range(3):
        b.train_step(s)
    b.save(2)
    c = Trainer(_args(tmp_path / "b", 6, extra=["--resume_path", b.log_dir]))
    c._resume_from_checkpoint()
    assert c.start_step == 3
    loss_c = c.train_step(3)["loss"].item()
    assert abs(loss_c - losses_a[3]) < 1e-6 * max(1.0, abs(losses_a[3])), (loss_c, losses_a)
    for (n, pa), (_, pc) in zip(a.raw_model.state_dict().items(), c.raw_model.state_dict().items()):
        assert torch.allclose(pa, pc, atol=1e-7), n


@pytest.mark.skipif(not ref_oracle.available(), reason="reference not installed under baseline/_ref")
def test_checkpoint_files_load_in_reference_loader(tmp_path, no_dist_env):
    """The reference's load_model_state_dict_for_training reads this framework's files (same
    names, key schema, fp32 tensors and meta), and the tensors round-trip exactly."""
    from tinytron_b200.training import checkpoint as ck
    from tinytron_b200.training.trainer import Trainer

    tr = Trainer(_args(tmp_path, 4))
    tr.train_step(0)
    tr.save(1)
    prefix = os.path.join(tr.log_dir, "00001")
    meta = torch.load(ck.checkpoint_meta_path(prefix), map_location="cpu", weights_only=False)
    ours = tr.raw_model.state_dict()
    ref_oracle.ensure_gloo_world1(port=29613)
    with ref_oracle.cpu_reference():
        from tinytron.distributed import parallel_state
        from tinytron.model.config import ModelConfig as RefCfg
        from tinytron.training import checkpoint as ref_ck
        from tinytron.training.config import ParallelConfig

        parallel_state.initialize_model_parallel(ParallelConfig(sep_size=1))
        rcfg = RefCfg(**{k: v for k, v in tr.config.model.__dict__.items() if k in RefCfg.__dataclass_fields__})
        sd = ref_ck.load_model_state_dict_for_training(prefix, rcfg, 0, meta)
        assert ref_ck.find_latest_checkpoint_prefix(tr.log_dir) == prefix
    assert set(sd) == set(ours)
    for k, v in ours.items():
        assert sd[k].dtype == torch.float32 and torch.equal(sd[k], v.cpu()), k
