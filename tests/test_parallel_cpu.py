"""Multi-rank semantics on CPU (gloo): SEP training (Ulysses attention + expert-parallel
MoE), head-parallel KV-cache decode and DP + ZeRO-1 must reproduce single-process
results for the same weights and data."""
import os
import socket
import tempfile

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from tinytron_b200.models import GPT, ModelConfig


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _entry(rank, world, port, fn, args):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    for k in ("RANK", "WORLD_SIZE", "LOCAL_RANK"):
        os.environ.pop(k, None)
    torch.set_num_threads(1)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        fn(rank, world, *args)
    finally:
        from tinytron_b200.parallel import parallel_state

        parallel_state.destroy_model_parallel()
        dist.destroy_process_group()


def spawn(fn, world, *args):
    mp.spawn(_entry, args=(world, _port(), fn, args), nprocs=world, join=True)


def cfg(**kw):
    base = dict(block_size=64, vocab_size=128, num_layer=2, num_attention_heads=4, num_key_value_heads=2,
                hidden_size=64, intermediate_size=96, init_std=0.02, seed=11)
    base.update(kw)
    return ModelConfig(**base)


def data(B=2, T=32, V=128, seed=5):
    g = torch.Generator().manual_seed(seed)
    x = torch.randint(0, V, (B, T), generator=g)
    y = torch.randint(0, V, (B, T), generator=g)
    return x, y


# ---------------------------------------------------------------- SEP training
def _sep_worker(rank, world, c, out_dir):
    from tinytron_b200.models.gpt import EXPERT_LOCAL_PARAM_SUFFIXES
    from tinytron_b200.parallel import allreduce_non_expert_grads_across_sp, parallel_state

    parallel_state.initialize_model_parallel(sep_size=world)
    torch.manual_seed(0)
    m = GPT(c, device="cpu")
    x, y = data(V=c.vocab_size)
    T = x.size(1) // world
    _, loss, ll = m(x[:, rank * T:(rank + 1) * T], y[:, rank * T:(rank + 1) * T])
    loss.backward()
    allreduce_non_expert_grads_across_sp(m, parallel_state.get_sp_group(), world, EXPERT_LOCAL_PARAM_SUFFIXES)
    torch.save({"ll": ll.item(), "grads": {n: p.grad.clone() for n, p in m.named_parameters()}},
               os.path.join(out_dir, f"r{rank}.pt"))


@pytest.mark.parametrize("kv,moe", [(2, False), (1, False), (2, True)])
def test_sep2_training_matches_single_rank(kv, moe):
    extra = dict(use_moe=True, num_experts=4, num_experts_per_tok=2, moe_intermediate_size=32,
                 moe_balance_loss_weight=0.01) if moe else {}
    c = cfg(num_key_value_heads=kv, **extra)
    with tempfile.TemporaryDirectory() as td:
        spawn(_sep_worker, 2, c, td)
        res = [torch.load(os.path.join(td, f"r{r}.pt")) for r in range(2)]
    full = GPT(c, device="cpu")
    x, y = data(V=c.vocab_size)
    _, loss, ll = full(x, y)
    loss.backward()
    for r in range(2):
        assert abs(res[r]["ll"] - ll.item()) < 1e-5
        for n, p in full.named_parameters():
            g = res[r]["grads"][n]
            if n.endswith(("experts_gate_weights", "experts_up_weights", "experts_down_weights")):
                ref = p.grad[r * 2:(r + 1) * 2]
            else:
                ref = p.grad
            assert torch.allclose(g, ref, atol=2e-5, rtol=1e-3), (r, n, (g - ref).abs().max())


# ---------------------------------------------------------------- head-parallel decode
def _decode_worker(rank, world, c, out_dir):
    from tinytron_b200.parallel import parallel_state

    parallel_state.initialize_model_parallel(sep_size=world)
    m = GPT(c, device="cpu").eval()
    x, _ = data(B=2, T=12, V=c.vocab_size)
    with torch.no_grad():
        l1, kv = m(x, use_cache=True)
        nxt = x[:, :1]
        l2, _ = m(nxt, use_cache=True, past_key_values=kv, position_offset=12)
    torch.save({"l1": l1, "l2": l2}, os.path.join(out_dir, f"r{rank}.pt"))


@pytest.mark.parametrize("kv,moe", [(2, False), (1, False), (2, True)])
def test_sep2_head_parallel_decode_matches_single_rank(kv, moe):
    extra = dict(use_moe=True, num_experts=4, num_experts_per_tok=2, moe_intermediate_size=32) if moe else {}
    c = cfg(num_key_value_heads=kv, **extra)
    with tempfile.TemporaryDirectory() as td:
        spawn(_decode_worker, 2, c, td)
        res = [torch.load(os.path.join(td, f"r{r}.pt")) for r in range(2)]
    m = GPT(c, device="cpu").eval()
    x, _ = data(B=2, T=12, V=c.vocab_size)
    with torch.no_grad():
        l1, kv_ = m(x, use_cache=True)
        l2, _ = m(x[:, :1], use_cache=True, past_key_values=kv_, position_offset=12)
    for r in range(2):
        assert torch.allclose(res[r]["l1"], l1, atol=1e-5)
        assert torch.allclose(res[r]["l2"], l2, atol=1e-5)


def _sample_worker(rank, world, c, out_dir):
    from tinytron_b200.inference import InferenceEngine
    from tinytron_b200.parallel import parallel_state

    parallel_state.initialize_model_parallel(sep_size=world)
    eng = InferenceEngine(c, device="cpu", use_paged_kv_cache=False)
    torch.manual_seed(100 + rank)  # ranks' own RNG streams differ on purpose
    x, _ = data(B=3, T=8, V=c.vocab_size)
    toks, info = eng.generate(x, 10, temperature=1.0, top_k=20, return_logprobs=True)
    torch.save({"toks": toks, "lp": info["token_log_probs"]}, os.path.join(out_dir, f"r{rank}.pt"))


def test_sep2_temperature_sampling_is_replicated_across_ranks():
    """Head-parallel ranks hold identical logits; with temperature > 0 they must also draw
    identical tokens (one seed sent by the group's first rank), or their KV caches would
    diverge after the first sampled step."""
    c = cfg()
    with tempfile.TemporaryDirectory() as td:
        spawn(_sample_worker, 2, c, td)
        res = [torch.load(os.path.join(td, f"r{r}.pt")) for r in range(2)]
    assert torch.equal(res[0]["toks"], res[1]["toks"])
    assert torch.allclose(res[0]["lp"], res[1]["lp"], atol=1e-6)
    assert res[0]["toks"].shape == (3, 18)


# ---------------------------------------------------------------- DP + ZeRO-1
def _dp_worker(rank, world, c, out_dir):
    from tinytron_b200.parallel import parallel_state
    from tinytron_b200.parallel.buffers import FlatParams
    from tinytron_b200.parallel.zero1 import FlatZeRO1

    parallel_state.initialize_model_parallel(sep_size=1)
    m = GPT(c, device="cpu")
    flat = FlatParams(m, pad_to_multiple=64 * world, with_bf16=False)
    opt = FlatZeRO1(flat, dp_group=parallel_state.get_dp_group(), lr=1e-2, weight_decay=0.1)
    x, y = data(B=4, V=c.vocab_size)
    for step in range(3):
        flat.zero_grad()
        _, loss, _ = m(x[rank * 2:(rank + 1) * 2], y[rank * 2:(rank + 1) * 2])
        loss.backward()
        for p in flat.params:
            p.__dict__["main_grad"].add_(p.grad)
            p.grad = None
        opt.reduce_gradients()
        norm, coef = opt.grad_norm_and_coef(1.0)
        opt.step(grad_scale=coef)
    torch.save({n: p.detach().clone() for n, p in m.named_parameters()}, os.path.join(out_dir, f"r{rank}.pt"))


def test_dp2_zero1_matches_single_rank_adamw():
    c = cfg()
    with tempfile.TemporaryDirectory() as td:
        spawn(_dp_worker, 2, c, td)
        res = [torch.load(os.path.join(td, f"r{r}.pt")) for r in range(2)]
    m = GPT(c, device="cpu")
    opt = torch.optim.AdamW(m.parameters(), lr=1e-2, weight_decay=0.1, betas=(0.9, 0.95), eps=1e-8)
    x, y = data(B=4, V=c.vocab_size)
    for step in range(3):
        opt.zero_grad()
        _, loss, _ = m(x, y)
        loss.backward()
        m.clip_grad_norm(1.0)
        opt.step()
    for n, p in m.named_parameters():
        for r in range(2):
            assert torch.allclose(res[r][n], p.detach(), atol=2e-5, rtol=1e-4), (n, r)


def test_grad_bucket_plan_tiles_buffer_and_interleaves_ownership():
    from tinytron_b200.parallel.zero1 import plan_grad_buckets

    offsets = [0, 64 * 10, 64 * 500, 64 * 900, 64 * 2000, 64 * 2100]
    numel = 64 * 2400
    for dp in (1, 2, 4, 8, 16):
        per_rank = []
        for r in range(dp):
            buckets, slices, state = plan_grad_buckets(offsets, numel, 64 * 700 * 4, dp, r)
            assert buckets[0][1] == numel and buckets[-1][0] == 0  # reverse order, tiles [0, numel)
            assert all(buckets[i][0] == buckets[i + 1][1] for i in range(len(buckets) - 1))
            assert all(lo in offsets or lo == 0 for lo, _ in buckets)  # whole parameters
            assert state[-1][1] == numel // dp and all(s1 - s0 == hi - lo for (s0, s1), (lo, hi) in zip(state, slices))
            per_rank.append(slices)
        cover = sorted(sl for sls in per_rank for sl in sls)  # the ranks' slices tile the buffer
        assert cover[0][0] == 0 and cover[-1][1] == numel
        assert all(cover[i][1] == cover[i + 1][0] for i in range(len(cover) - 1))


# ---------------------------------------------------------------- reference-compatible ZeRO-1 wrapper
def _distopt_worker(rank, world, c, out_dir, impl):
    import ref_oracle

    from tinytron_b200.parallel import parallel_state

    parallel_state.initialize_model_parallel(sep_size=1)
    torch.manual_seed(0)
    m = GPT(c, device="cpu")
    base = torch.optim.AdamW(m.parameters(), lr=1e-2, weight_decay=0.1, betas=(0.9, 0.95), eps=1e-8)
    if impl == "reference":
        with ref_oracle.cpu_reference():
            from tinytron.distributed import DistributedOptimizer
    else:
        from tinytron_b200.parallel import DistributedOptimizer
    opt = DistributedOptimizer(base, dist.group.WORLD)
    x, y = data(B=4, V=c.vocab_size)
    for step in range(3):
        opt.zero_grad()
        _, loss, _ = m(x[rank * 2:(rank + 1) * 2], y[rank * 2:(rank + 1) * 2])
        loss.backward()
        for p in m.parameters():  # data-parallel gradient mean, as the trainers do before step()
            dist.all_reduce(p.grad)
            p.grad /= world
        opt.step()
    torch.save({n: p.detach().clone() for n, p in m.named_parameters()}, os.path.join(out_dir, f"{impl}{rank}.pt"))


def test_distributed_optimizer_matches_reference_and_adamw():
    """The reference-compatible ZeRO-1 wrapper (each rank updates the tensors it owns and
    broadcasts them) gives the reference wrapper's parameters, equal on both ranks and
    equal to single-process AdamW on the full batch."""
    import ref_oracle

    if not ref_oracle.available():
        pytest.skip("reference not installed under baseline/_ref")
    c = cfg()
    with tempfile.TemporaryDirectory() as td:
        for impl in ("ours", "reference"):
            spawn(_distopt_worker, 2, c, td, impl)
        res = {(i, r): torch.load(os.path.join(td, f"{i}{r}.pt")) for i in ("ours", "reference") for r in range(2)}
    m = GPT(c, device="cpu")
    opt = torch.optim.AdamW(m.parameters(), lr=1e-2, weight_decay=0.1, betas=(0.9, 0.95), eps=1e-8)
    x, y = data(B=4, V=c.vocab_size)
    for step in range(3):
        opt.zero_grad()
        loss = sum(m(x[r * 2:(r + 1) * 2], y[r * 2:(r + 1) * 2])[1] for r in range(2)) / 2
        loss.backward()
        opt.step()
    for n, p in m.named_parameters():
        for r in range(2):
            assert torch.equal(res[("ours", r)][n], res[("ours", 0)][n]), (n, r)
            assert torch.allclose(res[("ours", r)][n], res[("reference", r)][n], atol=1e-6), (n, r)
            assert torch.allclose(res[("ours", r)][n], p.detach(), atol=2e-5, rtol=1e-4), (n, r)


# ---------------------------------------------------------------- public collective functions
def _collectives_worker(rank, world, out_dir):
    import ref_oracle

    from tinytron_b200.parallel import ep_all_to_all, ep_all_to_all_no_grad, ulysses_all_to_all

    with ref_oracle.cpu_reference():
        from tinytron.distributed import ep_all_to_all as r_ep
        from tinytron.distributed import ep_all_to_all_no_grad as r_ep_ng
        from tinytron.distributed import ulysses_all_to_all as r_ul
    g = torch.Generator().manual_seed(rank)
    group = dist.group.WORLD
    res = {}
    x = torch.randn(world * 3, 5, generator=g)
    for tag, fn in (("ours", ulysses_all_to_all), ("ref", r_ul)):
        xi = x.clone().requires_grad_(True)
        y = fn(xi, group)
        (y * torch.arange(y.numel(), dtype=torch.float32).view_as(y)).sum().backward()
        res[f"ul_{tag}"], res[f"ul_grad_{tag}"] = y.detach(), xi.grad
    # uneven splits, including an empty one: rank r sends (r + c) % 3 rows to rank c
    in_splits = [(rank + c) % 3 for c in range(world)]
    out_splits = [(c + rank) % 3 for c in range(world)]
    h = torch.randn(sum(in_splits), 4, generator=g)
    for tag, fn, fn_ng in (("ours", ep_all_to_all, ep_all_to_all_no_grad), ("ref", r_ep, r_ep_ng)):
        hi = h.clone().requires_grad_(True)
        y = fn(hi, in_splits, out_splits, group)
        (y * (1 + torch.arange(y.numel(), dtype=torch.float32).view_as(y))).sum().backward()
        res[f"ep_{tag}"], res[f"ep_grad_{tag}"] = y.detach(), hi.grad
        res[f"epng_{tag}"] = fn_ng(h.clone(), in_splits, out_splits, group)
    # SP gradient sum of the non-expert parameters (expert gradients stay local), with a
    # bucket size that splits the parameters over several buckets
    from tinytron_b200.models.gpt import EXPERT_LOCAL_PARAM_SUFFIXES
    from tinytron_b200.parallel import allreduce_non_expert_grads_across_sp as ours_sp

    with ref_oracle.cpu_reference():
        from tinytron.distributed import allreduce_non_expert_grads_across_sp as ref_sp
    c = cfg(use_moe=True, num_experts=3, num_experts_per_tok=1, moe_intermediate_size=16)
    for tag, fn in (("ours", ours_sp), ("ref", ref_sp)):
        torch.manual_seed(0)
        m = GPT(c, device="cpu")
        gg = torch.Generator().manual_seed(100 + rank)
        for p in m.parameters():
            p.grad = torch.randn(p.shape, generator=gg)
        fn(m, group, world, EXPERT_LOCAL_PARAM_SUFFIXES, bucket_size_mb=0)
        res[f"sp_{tag}"] = {n: p.grad.clone() for n, p in m.named_parameters()}
    torch.save(res, os.path.join(out_dir, f"r{rank}.pt"))


def test_public_collectives_match_reference():
    """ulysses_all_to_all, ep_all_to_all (uneven splits with empty ones) and
    ep_all_to_all_no_grad give the reference's outputs and input gradients, and
    allreduce_non_expert_grads_across_sp its gradients (expert ones left local)."""
    import ref_oracle

    if not ref_oracle.available():
        pytest.skip("reference not installed under baseline/_ref")
    with tempfile.TemporaryDirectory() as td:
        spawn(_collectives_worker, 3, td)
        res = [torch.load(os.path.join(td, f"r{r}.pt")) for r in range(3)]
    for r in range(3):
        for k in ("ul", "ul_grad", "ep", "ep_grad", "epng"):
            assert torch.equal(res[r][f"{k}_ours"], res[r][f"{k}_ref"]), (r, k)
        for n, g in res[r]["sp_ref"].items():
            assert torch.allclose(res[r]["sp_ours"][n], g, atol=1e-6), (r, n)


# ---------------------------------------------------------------- live training -> inference reshard
def _live_reshard_worker(rank, world, out_dir):
    from dataclasses import replace

    import ref_oracle
    from tinytron_b200.bridge import (build_tinytron_canonical_layout, build_tinytron_inference_layout,
                                      build_tinytron_training_layout, current_tinytron_parallel_spec,
                                      current_tinytron_placement, distributed_training_state_dict_to_local_inference)
    from tinytron_b200.bridge.layout import to_torch_slices
    from tinytron_b200.parallel import parallel_state

    c = cfg(use_moe=True, num_experts=4, num_experts_per_tok=2, moe_intermediate_size=32)
    parallel_state.initialize_model_parallel(sep_size=world)
    canon = build_tinytron_canonical_layout(c)
    g = torch.Generator().manual_seed(0)  # the same full tensors on every rank
    full = {s.param_name: torch.randn(s.global_shape, generator=g) for s in canon.local_shards(canon.placements()[0])}
    train = build_tinytron_training_layout(c, current_tinytron_parallel_spec("training"))
    mine = current_tinytron_placement(train)
    sd = {s.param_name: full[s.param_name][to_torch_slices(s.global_slices)].clone() for s in train.local_shards(mine)}
    icfg = replace(c, inference_shard_qkv=True)
    res = {"p2p": distributed_training_state_dict_to_local_inference(sd, icfg, use_p2p=True),
           "bcast": distributed_training_state_dict_to_local_inference(sd, icfg, use_p2p=False)}
    dst = build_tinytron_inference_layout(icfg, current_tinytron_parallel_spec("inference"), shard_qkv=True)
    res["want"] = {s.param_name: full[s.param_name][to_torch_slices(s.global_slices)]
                   for s in dst.local_shards(current_tinytron_placement(dst))}
    with ref_oracle.cpu_reference():
        from tinytron.bridge import distributed_training_state_dict_to_local_inference as ref_fn
        from tinytron.distributed import parallel_state as ref_ps
        from tinytron.model.config import ModelConfig as RefCfg
        from tinytron.training.config import ParallelConfig

        ref_ps.initialize_model_parallel(ParallelConfig(sep_size=world))
        rcfg = RefCfg(**{k: v for k, v in icfg.__dict__.items() if k in RefCfg.__dataclass_fields__})
        res["ref"] = ref_fn(sd, rcfg)
    torch.save(res, os.path.join(out_dir, f"r{rank}.pt"))


def test_live_reshard_matches_reference():
    """Every rank's SEP=2 training shard -> its q/k/v-sharded inference shard over gloo:
    the packed per-rank-pair transfer and the broadcast mode both give the reference
    bridge's tensors, which are the full tensors' slices."""
    import ref_oracle

    if not ref_oracle.available():
        pytest.skip("reference not installed under baseline/_ref")
    with tempfile.TemporaryDirectory() as td:
        spawn(_live_reshard_worker, 2, td)
        res = [torch.load(os.path.join(td, f"r{r}.pt")) for r in range(2)]
    for r in range(2):
        want = res[r]["want"]
        assert any("experts" in k for k in want) and any("q_proj" in k for k in want)
        for mode in ("p2p", "bcast", "ref"):
            got = res[r][mode]
            assert set(got) == set(want), (r, mode, sorted(set(got) ^ set(want)))
            for k in want:
                assert torch.equal(got[k], want[k]), (r, mode, k)


# ---------------------------------------------------------------- parallel_state getters
_GETTERS = ["dp_world_size", "dp_rank", "dp_global_rank", "sep_world_size", "sep_rank", "sep_global_rank",
            "sp_world_size", "sp_rank", "sp_global_rank", "ep_world_size", "ep_rank", "ep_global_rank",
            "dp_sp_world_size", "dp_sp_rank", "dp_sp_global_rank"]


def _state_worker(rank, world, out_dir):
    import ref_oracle
    from tinytron_b200.parallel import parallel_state as ours

    def snapshot(ps):
        out = {}
        for n in _GETTERS:
            fn = getattr(ps, f"get_{n}")
            out[n] = fn(0) if n.endswith("global_rank") else fn()
        for grp in ("dp", "sep", "sp", "ep", "dp_sp"):
            out[f"{grp}_members"] = sorted(dist.get_process_group_ranks(getattr(ps, f"get_{grp}_group")()))
        return out

    ours.initialize_model_parallel(sep_size=2)
    res = {"ours": snapshot(ours)}
    with ref_oracle.cpu_reference():
        from tinytron.distributed import parallel_state as ref
        from tinytron.training.config import ParallelConfig

        ref.initialize_model_parallel(ParallelConfig(sep_size=2))
        res["ref"] = snapshot(ref)
    torch.save(res, os.path.join(out_dir, f"r{rank}.pt"))


def test_parallel_state_getters_match_reference():
    """Four gloo ranks at SEP=2: every rank/world-size getter and the member ranks of the
    DP, SEP (SP, EP) and DP x SEP groups equal the reference's."""
    import ref_oracle

    if not ref_oracle.available():
        pytest.skip("reference not installed under baseline/_ref")
    with tempfile.TemporaryDirectory() as td:
        spawn(_state_worker, 4, td)
        res = [torch.load(os.path.join(td, f"r{r}.pt")) for r in range(4)]
    for r in range(4):
        assert res[r]["ours"] == res[r]["ref"], (r, res[r])
    assert res[1]["ours"]["sep_members"] == [0, 1] and res[1]["ours"]["dp_members"] == [1, 3]
