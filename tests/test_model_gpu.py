"""Full model on the sm_100a path vs the same model's CPU fp32 path (same weights)."""
import pytest
import torch

from tinytron_b200.models import GPT, ModelConfig
from tinytron_b200.parallel.buffers import FlatParams

pytestmark = pytest.mark.gpu


def _cfg(**kw):
    base = dict(block_size=512, vocab_size=1024, num_layer=2, num_attention_heads=2, num_key_value_heads=1,
                hidden_size=256, intermediate_size=512, init_std=0.02, seed=3)
    base.update(kw)
    return ModelConfig(**base)


def _rel(a, b):
    return ((a.float() - b.float()).norm() / (b.float().norm() + 1e-12)).item()


@pytest.mark.parametrize("flat", [False, True])
def test_gpu_forward_backward_matches_cpu_fp32(flat):
    cfg = _cfg()
    cpu = GPT(cfg, device="cpu")
    gpu = GPT(cfg, device="cuda")
    gpu.load_state_dict(cpu.state_dict())
    fp = FlatParams(gpu) if flat else None
    x = torch.randint(0, cfg.vocab_size, (2, 256))
    y = torch.randint(0, cfg.vocab_size, (2, 256))
    y[1, :17] = -100
    _, lc, llc = cpu(x, y)
    lc.backward()
    _, lg, llg = gpu(x.cuda(), y.cuda())
    lg.backward()
    torch.cuda.synchronize()
    assert abs(lg.item() - lc.item()) < 2e-2 * abs(lc.item())
    assert abs(llg.item() - llc.item()) < 2e-2 * abs(llc.item())
    for (n, pc), (_, pg) in zip(cpu.named_parameters(), gpu.named_parameters()):
        g = pg.__dict__["main_grad"] if flat else pg.grad
        assert g is not None, n
        assert _rel(g.cpu(), pc.grad) < 6e-2, (n, _rel(g.cpu(), pc.grad))
    from tinytron_b200.ops import check_status

    check_status()


def test_gpu_logits_and_cached_decode():
    cfg = _cfg()
    cpu = GPT(cfg, device="cpu").eval()
    gpu = GPT(cfg, device="cuda").eval()
    gpu.load_state_dict(cpu.state_dict())
    x = torch.randint(0, cfg.vocab_size, (2, 64))
    with torch.no_grad():
        lc = cpu(x)
        lg = gpu(x.cuda())
        assert _rel(lg.cpu(), lc) < 3e-2
        lc1, kvc = cpu(x, use_cache=True)
        lg1, kvg = gpu(x.cuda(), use_cache=True)
        nxt = torch.randint(0, cfg.vocab_size, (2, 1))
        lc2, _ = cpu(nxt, use_cache=True, past_key_values=kvc, position_offset=64)
        lg2, _ = gpu(nxt.cuda(), use_cache=True, past_key_values=kvg, position_offset=64)
        assert _rel(lg2.cpu(), lc2) < 3e-2


def test_gpu_trainer_steps(tmp_path, monkeypatch):
    for k in ("RANK", "WORLD_SIZE", "LOCAL_RANK", "MASTER_ADDR"):
        monkeypatch.delenv(k, raising=False)
    from tinytron_b200.training import build_config, parse_args
    from tinytron_b200.training.trainer import Trainer

    argv = ["--use_mock_data", "--deterministic", "--mock_data_num_samples", "4", "--log_dir", str(tmp_path),
            "--total_batch_size", str(4 * 256 * 2), "--batch_size", "4", "--seq_len", "256", "--max_steps", "10",
            "--warmup_steps", "2", "--max_lr", "3e-3", "--num_layer", "2", "--hidden_size", "256",
            "--num_attention_heads", "2", "--num_key_value_heads", "1", "--intermediate_size", "512",
            "--vocab_size", "1024", "--block_size", "512", "--init_std", "0.02"]
    tr = Trainer(build_config(parse_args(argv)))
    tr.train()
    losses = [tr.results[s]["loss"].item() for s in sorted(tr.results)]
    assert all(l == l for l in losses)
    assert losses[-1] < losses[0] - 0.1, losses
