"""Packed scalar all-reduce (one collective for every per-micro-step statistic) on gloo
ranks, and the executed-FLOP count behind the MFU figures."""
import os
import socket
import tempfile

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _scalars_worker(rank, world, port, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.set_num_threads(1)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from tinytron_b200.parallel.scalars import (_MAX_FLOATS, all_reduce_scalars, rank_slot_vector,
                                                    release_scalar_reducers)

        group = dist.new_group(list(range(world)))
        # odd length (padded to a multiple of 4 inside), 2-D shape kept
        vec = torch.arange(6, dtype=torch.float32).view(2, 3) * (rank + 1)
        summed = all_reduce_scalars(vec, group)
        slots = all_reduce_scalars(rank_slot_vector(torch.tensor(10.0 + rank), rank, world), group)
        too_long = None
        try:
            all_reduce_scalars(torch.zeros(_MAX_FLOATS + 1), group)
        except ValueError as e:
            too_long = str(e)
        single = all_reduce_scalars(vec, None)  # no group: a copy
        release_scalar_reducers()
        torch.save({"summed": summed, "vec": vec, "slots": slots, "too_long": too_long, "single": single},
                   os.path.join(out_dir, f"r{rank}.pt"))
    finally:
        dist.destroy_process_group()


def test_packed_scalar_all_reduce_gloo():
    world = 3
    with tempfile.TemporaryDirectory() as td:
        mp.spawn(_scalars_worker, args=(world, _port(), td), nprocs=world, join=True)
        res = [torch.load(os.path.join(td, f"r{r}.pt")) for r in range(world)]
    want = torch.arange(6, dtype=torch.float32).view(2, 3) * sum(r + 1 for r in range(world))
    for r in range(world):
        assert res[r]["summed"].shape == (2, 3)
        assert torch.equal(res[r]["summed"], want)
        assert torch.equal(res[r]["vec"], torch.arange(6, dtype=torch.float32).view(2, 3) * (r + 1))  # input intact
        assert torch.equal(res[r]["slots"], torch.tensor([10.0, 11.0, 12.0]))  # one slot per rank
        assert res[r]["too_long"] is not None and "at most" in res[r]["too_long"]
        assert torch.equal(res[r]["single"], res[r]["vec"])


@pytest.mark.parametrize("moe", [False, True])
def test_training_flops_match_parameter_count(moe):
    """3 x forward; forward = 2 x (matmul parameters per token) x tokens plus the causal
    attention products (QK^T and PV over half of the T x T scores)."""
    from tinytron_b200.models import ModelConfig
    from tinytron_b200.utils.flops import training_flops_per_microstep

    kw = dict(block_size=4096, vocab_size=50304, num_layer=24, num_attention_heads=16, num_key_value_heads=4,
              hidden_size=2048, intermediate_size=5504)
    if moe:
        kw.update(use_moe=True, num_experts=64, num_experts_per_tok=8, moe_intermediate_size=1408)
    c = ModelConfig(**kw)
    B, T, sp = 4, 4096, 2
    D, hd, L = 2048, 128, 24
    tok = B * T
    per_layer = D * (16 + 2 * 4) * hd + D * D  # qkv + output projection
    per_layer += (8 * 3 * D * 1408 + D * 64) if moe else 3 * D * 5504  # active experts + router, or dense MLP
    fwd = 2 * tok * (L * per_layer + D * 50304) + L * 2 * tok * (T * sp) * D
    assert training_flops_per_microstep(c, B, T, sp) == pytest.approx(3 * fwd, rel=1e-12)
