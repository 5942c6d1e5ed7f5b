"""Muon: CPU parity with the unmodified reference optimizer, and the tcgen05
Newton-Schulz path vs the fp32 iteration on GPU."""
import pytest
import torch

import ref_oracle


def _params(seed):
    g = torch.Generator().manual_seed(seed)
    return [torch.randn(64, 48, generator=g), torch.randn(32, 96, generator=g), torch.randn(48, generator=g)]


@pytest.mark.skipif(not ref_oracle.available(), reason="reference not installed under baseline/_ref")
def test_muon_matches_reference_on_cpu():
    """Muon group: optimizer steps match the reference Muon.  Adam group: the update
    function matches (the reference's Muon cannot build an Adam group: its key check
    rejects both with and without ``use_adam``)."""
    from tinytron_b200.optim import Muon
    from tinytron_b200.optim.muon import adam_update

    with ref_oracle.cpu_reference():
        from tinytron.optim.muon import Muon as RefMuon
        from tinytron.optim.muon import adam_update as ref_adam_update
    ours = [torch.nn.Parameter(p.clone()) for p in _params(0)[:2]]
    ref = [torch.nn.Parameter(p.clone()) for p in _params(0)[:2]]
    opt_o = Muon([{"params": ours, "use_muon": True, "lr": 0.02, "momentum": 0.95, "weight_decay": 0.1}])
    opt_r = RefMuon([{"params": ref, "use_muon": True, "lr": 0.02, "momentum": 0.95, "weight_decay": 0.1}])
    g = torch.Generator().manual_seed(1)
    for _ in range(3):
        grads = [torch.randn(p.shape, generator=g) for p in ours]
        for p, q, gr in zip(ours, ref, grads):
            p.grad = gr.clone()
            q.grad = gr.clone()
        opt_o.step()
        opt_r.step()
    for p, q in zip(ours, ref):
        assert torch.allclose(p, q, atol=1e-5, rtol=1e-5), (p - q).abs().max()
    gr = torch.randn(48, generator=g)
    b1o, b2o, b1r, b2r = (torch.zeros(48) for _ in range(4))
    for step in (1, 2):
        uo = adam_update(gr.clone(), b1o, b2o, step, (0.9, 0.95), 1e-10)
        ur = ref_adam_update(gr.clone(), b1r, b2r, step, (0.9, 0.95), 1e-10)
        assert torch.allclose(uo, ur)


@pytest.mark.gpu
@pytest.mark.parametrize("shape", [(256, 2048), (2048, 2048), (1024, 384), (5504, 2048)])
def test_newton_schulz_tcgen05_matches_fp32(shape):
    from tinytron_b200.optim.muon import NS_COEFFS, zeropower_via_newtonschulz5

    g = torch.Generator(device="cuda").manual_seed(0)
    G = torch.randn(*shape, device="cuda", generator=g)
    out = zeropower_via_newtonschulz5(G, 5)
    a, b, c = NS_COEFFS
    X = G.double()
    if X.size(0) > X.size(1):
        X = X.mT
    X = X / (X.norm() + 1e-7)
    for _ in range(5):
        A = X @ X.mT
        X = a * X + (b * A + c * A @ A) @ X
    if G.size(0) > G.size(1):
        X = X.mT
    err = ((out.double() - X).norm() / X.norm()).item()
    assert out.shape == G.shape and err < 3e-2, err


# ----------------------------------------------------------------------------- fused NS GEMMs
@pytest.mark.gpu
@pytest.mark.parametrize("r,n", [(256, 2048), (384, 1024), (2048, 2048), (200, 520)])
def test_gemm_axpby_symmetric_and_fused_epilogue(r, n):
    from tinytron_b200.ops import _ext, check_status

    C = _ext.load()
    g = torch.Generator(device="cuda").manual_seed(r + n)
    X = (torch.randn(r, n, device="cuda", generator=g) / n ** 0.5).bfloat16()
    A = torch.empty(r, r, device="cuda", dtype=torch.bfloat16)
    C.gemm_axpby(X, X, A, False, 1.0, None, 0.0, True)  # symmetric X X^T
    Xf = X.float()
    ref_A = Xf @ Xf.t()
    B = torch.empty_like(A)
    C.gemm_axpby(A, A, B, False, 2.0315, A, -4.775, True)  # c A^2 + b A
    Af = A.float()
    ref_B = 2.0315 * Af @ Af + -4.775 * Af
    out = torch.empty_like(X)
    C.gemm_axpby(B, X, out, True, 1.0, X, 3.4445, False)  # B X + a X
    ref_out = B.float() @ Xf + 3.4445 * Xf
    torch.cuda.synchronize()
    check_status()
    rel = lambda a, b: ((a.float() - b).norm() / b.norm()).item()  # noqa: E731
    assert rel(A, ref_A) < 1e-2 and torch.equal(A, A.t())
    assert rel(B, ref_B) < 1e-2 and torch.equal(B, B.t())
    assert rel(out, ref_out) < 1e-2


# ----------------------------------------------------------------------------- ZeRO-1 Muon
def _dist_muon_worker(rank, world, out_dir):
    import os

    import torch.distributed as dist

    from tinytron_b200.models import GPT, ModelConfig
    from tinytron_b200.optim import Muon
    from tinytron_b200.optim.muon import DistributedMuon
    from tinytron_b200.parallel.buffers import FlatParams

    cfg = ModelConfig(block_size=32, vocab_size=64, num_layer=2, num_attention_heads=4, num_key_value_heads=2,
                      hidden_size=32, intermediate_size=48, init_std=0.02, seed=5)

    def build():
        m = GPT(cfg, device="cpu")
        flat = FlatParams(m, with_bf16=False)
        mat = [p for n, p in m.named_parameters() if p.ndim == 2 and "wte" not in n and "lm_head" not in n]
        rest = [p for n, p in m.named_parameters() if not any(p is q for q in mat)]
        opt = Muon([{"params": mat, "use_muon": True, "lr": 0.02, "momentum": 0.95, "weight_decay": 0.1},
                    {"params": rest, "use_muon": False, "use_adam": True, "lr": 1e-3, "weight_decay": 0.1}])
        return m, flat, opt

    m, flat, opt = build()
    dopt = DistributedMuon(opt, flat, dense_group=dist.group.WORLD)
    owned = sum(len(g["params"]) for g in opt.param_groups)
    single_m, single_flat, single_opt = build()
    gen = torch.Generator().manual_seed(0)
    for step in range(3):
        grad = torch.randn(flat.numel, generator=gen)
        for f in (flat, single_flat):
            f.grad.copy_(grad)
            f.expose_grads()
        coef = torch.tensor(0.5)
        dopt.step(grad_scale=coef)
        single_opt.step(grad_scale=coef)
    torch.save({"diff": (flat.data - single_flat.data).abs().max().item(), "owned": owned,
                "total": sum(len(g["params"]) for g in single_opt.param_groups)},
               os.path.join(out_dir, f"r{rank}.pt"))


def test_distributed_muon_matches_single_rank(tmp_path):
    import os

    from test_parallel_cpu import spawn

    spawn(_dist_muon_worker, 2, str(tmp_path))
    r0, r1 = (torch.load(os.path.join(tmp_path, f"r{i}.pt")) for i in range(2))
    assert r0["diff"] < 1e-6 and r1["diff"] < 1e-6, (r0, r1)
    assert 0 < r0["owned"] < r0["total"] and r0["owned"] + r1["owned"] == r0["total"]


def test_trainer_with_muon_runs_cpu(tmp_path, monkeypatch):
    for k in ("RANK", "WORLD_SIZE", "LOCAL_RANK", "MASTER_ADDR"):
        monkeypatch.delenv(k, raising=False)
    from tinytron_b200.training import build_config, parse_args
    from tinytron_b200.training.trainer import Trainer

    argv = ["--use_mock_data", "--deterministic", "--mock_data_num_samples", "8", "--log_dir", str(tmp_path),
            "--total_batch_size", str(4 * 32), "--batch_size", "4", "--seq_len", "32", "--max_steps", "6",
            "--warmup_steps", "1", "--max_lr", "2e-2", "--min_lr", "2e-3", "--optimizer", "muon",
            "--num_layer", "2", "--hidden_size", "64", "--num_attention_heads", "4", "--num_key_value_heads", "2",
            "--intermediate_size", "96", "--vocab_size", "128", "--block_size", "32", "--backend", "gloo"]
    tr = Trainer(build_config(parse_args(argv)))
    tr.train()
    losses = [tr.results[s]["loss"].item() for s in sorted(tr.results)]
    assert all(torch.isfinite(torch.tensor(losses))) and losses[-1] < losses[0], losses


def _muon_trainer_rank(rank, world, port, tmp, out):
    import os

    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank), MASTER_ADDR="127.0.0.1",
                      MASTER_PORT=str(port))
    torch.set_num_threads(1)
    from tinytron_b200.training import build_config, parse_args
    from tinytron_b200.training.trainer import Trainer

    argv = ["--use_mock_data", "--deterministic", "--mock_data_num_samples", "8", "--log_dir", tmp,
            "--total_batch_size", str(4 * 32), "--batch_size", "4", "--seq_len", "32", "--max_steps", "4",
            "--warmup_steps", "1", "--max_lr", "2e-2", "--min_lr", "2e-3", "--optimizer", "muon", "--sep_size", "2",
            "--num_layer", "2", "--hidden_size", "64", "--num_attention_heads", "4", "--num_key_value_heads", "2",
            "--intermediate_size", "96", "--vocab_size", "128", "--block_size", "32", "--backend", "gloo"]
    tr = Trainer(build_config(parse_args(argv)))
    for s in range(3):
        tr.train_step(s)
    torch.save({"data": tr.flat.data.clone(), "loss": float(tr.one_step_results["loss"])},
               os.path.join(out, f"r{rank}.pt"))
    tr.close()


def test_trainer_with_distributed_muon_sep2_gloo(tmp_path):
    """SEP=2: each matrix is orthogonalised by one of the two ranks and broadcast; both
    ranks end with identical dense parameters."""
    import os

    import torch.multiprocessing as mp
    from test_rl_trainer import _port

    mp.spawn(_muon_trainer_rank, args=(2, _port(), str(tmp_path / "logs"), str(tmp_path)), nprocs=2, join=True)
    r0, r1 = (torch.load(os.path.join(tmp_path, f"r{i}.pt")) for i in range(2))
    assert torch.equal(r0["data"], r1["data"])
    assert abs(r0["loss"] - r1["loss"]) < 1e-6


@pytest.mark.gpu
@pytest.mark.parametrize("batch,r,n", [(3, 256, 2048), (4, 128, 384), (2, 200, 520)])
def test_gemm_axpby_batched(batch, r, n):
    """Stacked products in one launch equal the per-matrix products."""
    from tinytron_b200.ops import _ext, check_status

    C = _ext.load()
    g = torch.Generator(device="cuda").manual_seed(batch + r)
    X = (torch.randn(batch * r, n, device="cuda", generator=g) / n ** 0.5).bfloat16()
    A = torch.empty(batch * r, r, device="cuda", dtype=torch.bfloat16)
    C.gemm_axpby(X, X, A, False, 1.0, None, 0.0, True, batch)
    B = torch.empty_like(A)
    C.gemm_axpby(A, A, B, False, 2.0, A, -1.5, True, batch)
    out = torch.empty_like(X)
    C.gemm_axpby(B, X, out, True, 1.0, X, 0.75, False, batch)
    torch.cuda.synchronize()
    check_status()
    rel = lambda a, b: ((a.float() - b).norm() / b.norm()).item()  # noqa: E731
    for i in range(batch):
        x = X[i * r:(i + 1) * r].float()
        a = A[i * r:(i + 1) * r]
        assert rel(a, x @ x.t()) < 1e-2 and torch.equal(a, a.t())
        af = a.float()
        assert rel(B[i * r:(i + 1) * r], 2.0 * af @ af - 1.5 * af) < 1e-2
        assert rel(out[i * r:(i + 1) * r], B[i * r:(i + 1) * r].float() @ x + 0.75 * x) < 1e-2


@pytest.mark.gpu
def test_muon_batched_step_matches_cpu():
    """A Muon step over same-shape (batched, incl. tall) and odd-shape matrices on the GPU
    matches the CPU reference-math step to bf16 accuracy."""
    from tinytron_b200.optim import Muon

    g = torch.Generator().manual_seed(3)
    shapes = [(256, 512), (256, 512), (256, 512), (768, 256), (768, 256), (64, 96)]
    init = [torch.randn(s, generator=g) * 0.02 for s in shapes]
    grads = [torch.randn(s, generator=g) for s in shapes]
    res = {}
    for dev in ("cpu", "cuda"):
        ps = [torch.nn.Parameter(t.clone().to(dev)) for t in init]
        opt = Muon([{"params": ps, "use_muon": True, "lr": 0.02, "momentum": 0.95, "weight_decay": 0.1}])
        for _ in range(2):
            for p, gr in zip(ps, grads):
                p.grad = gr.clone().to(dev)
            opt.step()
        res[dev] = [p.detach().cpu() for p in ps]
    for a, b, t0 in zip(res["cpu"], res["cuda"], init):
        da, db = a - t0, b - t0
        assert ((da - db).norm() / da.norm()).item() < 3e-2


def _muon_moe_dp_rank(rank, world, port, tmp, out):
    import os

    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank), MASTER_ADDR="127.0.0.1",
                      MASTER_PORT=str(port))
    torch.set_num_threads(1)
    from tinytron_b200.training import build_config, parse_args
    from tinytron_b200.training.trainer import Trainer

    argv = ["--use_mock_data", "--deterministic", "--mock_data_num_samples", "16", "--log_dir", tmp,
            "--total_batch_size", str(2 * 32 * 2), "--batch_size", "2", "--seq_len", "32", "--max_steps", "4",
            "--warmup_steps", "1", "--max_lr", "2e-2", "--min_lr", "2e-3", "--optimizer", "muon",
            "--num_layer", "2", "--hidden_size", "64", "--num_attention_heads", "4", "--num_key_value_heads", "2",
            "--intermediate_size", "96", "--vocab_size", "128", "--block_size", "32", "--backend", "gloo",
            "--use_moe", "--num_experts", "4", "--num_experts_per_tok", "2", "--moe_intermediate_size", "32"]
    tr = Trainer(build_config(parse_args(argv)))
    for s in range(2):
        tr.train_step(s)
    owned = sum(len(g["params"]) for g in tr.raw_optimizer.param_groups)
    torch.save({"data": tr.flat.data.clone(), "owned": owned}, os.path.join(out, f"r{rank}.pt"))
    tr.close()


def test_trainer_with_distributed_muon_moe_dp2_gloo(tmp_path):
    """DP=2 with MoE: dense and expert matrices are split between the two replicas, and
    the broadcasts leave both replicas with identical parameters."""
    import os

    import torch.multiprocessing as mp
    from test_rl_trainer import _port

    mp.spawn(_muon_moe_dp_rank, args=(2, _port(), str(tmp_path / "logs"), str(tmp_path)), nprocs=2, join=True)
    r0, r1 = (torch.load(os.path.join(tmp_path, f"r{i}.pt")) for i in range(2))
    assert torch.equal(r0["data"], r1["data"])
    assert r0["owned"] > 0 and r1["owned"] > 0
