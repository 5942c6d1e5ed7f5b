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
    # every key the reference trainer writes into _meta.pt and reads back on resume
    assert {"config", "step", "this_step_results", "opt_part_assignment", "model_layout", "model_sharded",
            "model_shard_pattern", "sampler_state", "rng_state"} <= set(meta), sorted(meta)
    assert set(meta["sampler_state"]) >= {"epoch", "iter_idx"} and meta["step"] == 1
    assert meta["model_shard_pattern"].format(rank=0) == os.path.basename(ck.checkpoint_model_shard_path(prefix, 0))
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


def test_reference_checkpoint_files_load_here(tmp_path, no_dist_env):
    """The other direction: files written by the reference's own save functions (rank shard,
    full model, meta with its training layout) load through this framework's training and
    inference loaders, and the loaded model computes the reference model's logits."""
    from tinytron_b200.inference import checkpoint as icp
    from tinytron_b200.models import GPT, ModelConfig
    from tinytron_b200.parallel import parallel_state as ps
    from tinytron_b200.training import checkpoint as ck

    cfg = ModelConfig(block_size=64, vocab_size=256, num_layer=2, num_attention_heads=4, num_key_value_heads=2,
                      hidden_size=64, intermediate_size=96, init_std=0.02, seed=7)
    prefix = str(tmp_path / "00002")
    x = torch.randint(0, 256, (2, 16), generator=torch.Generator().manual_seed(1))
    ref_oracle.ensure_gloo_world1(port=29615)
    with ref_oracle.cpu_reference():
        from tinytron.distributed import parallel_state
        from tinytron.model import GPT as RefGPT
        from tinytron.model.config import ModelConfig as RefCfg
        from tinytron.training import checkpoint as ref_ck
        from tinytron.training.config import ParallelConfig

        parallel_state.initialize_model_parallel(ParallelConfig(sep_size=1))
        torch.manual_seed(0)
        rm = RefGPT(RefCfg(**{k: v for k, v in cfg.__dict__.items() if k in RefCfg.__dataclass_fields__})).eval()
        ref_ck.save_local_model_shard(rm, prefix, 0)
        ref_ck.save_rank0_legacy_model(rm, prefix)
        torch.save({"model_layout": ref_ck.model_layout_metadata(), "model_sharded": True,
                    "model_shard_pattern": "00002_model_rank{rank:05d}.pt"}, ref_ck.checkpoint_meta_path(prefix))
        with torch.no_grad():
            want = rm(x)
    own_state = not ps.model_parallel_is_initialized()
    if own_state:
        ps.initialize_model_parallel(sep_size=1)
    try:
        meta = torch.load(ck.checkpoint_meta_path(prefix), map_location="cpu", weights_only=False)
        assert ck.find_latest_checkpoint_prefix(str(tmp_path)) == prefix
        for sd in (ck.load_model_state_dict_for_training(prefix, cfg, 0, meta),
                   icp.load_model_state_dict_for_inference(ck.checkpoint_model_shard_path(prefix, 0), cfg),
                   icp.load_model_state_dict_for_inference(ck.checkpoint_model_path(prefix), cfg)):
            m = GPT(cfg, device="cpu").eval()
            m.load_state_dict(sd, strict=True)
            with torch.no_grad():
                assert torch.allclose(m(x), want, atol=1e-5)
    finally:
        if own_state:
            ps.destroy_model_parallel()
