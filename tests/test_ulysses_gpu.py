"""Fused Ulysses head<->sequence exchange (csrc/runtime/ulysses.cu) on the GPU.

One GPU: W emulated ranks (W heaps on one device).  Every rank's pack is launched before
any rank's exchange, so each exchange only waits for packs that have already finished.
The kernels' results are compared with the layout the attention expects, built with
plain tensor ops (kv heads routed unexpanded; gradients of shared kv heads summed).
Two GPUs: a 2-layer GPT at SEP=2 (forward + backward through the fused path) against
the same model at SEP=1.
"""
import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _ref_full(qkvs, B, T, Hq, Hkv, D, sp, r):
    """Rank r's [B * sp * T, W] buffer: its q heads and the kv heads they read, for every
    rank's token chunk in order."""
    from tinytron_b200.parallel.ulysses import kv_heads_for_rank

    hq_l = Hq // sp
    k0, k1 = kv_heads_for_rank(r, sp, Hq, Hkv)
    rows = []
    for c in range(sp):
        x = qkvs[c].view(B, T, Hq + 2 * Hkv, D)
        rows.append(torch.cat([x[:, :, r * hq_l:(r + 1) * hq_l], x[:, :, Hq + k0:Hq + k1],
                               x[:, :, Hq + Hkv + k0:Hq + Hkv + k1]], 2))
    return torch.stack(rows, 1).reshape(B * sp * T, -1)


@pytest.mark.parametrize("sp,Hq,Hkv", [(2, 16, 4), (4, 16, 4), (8, 16, 2), (4, 8, 8)])
def test_fused_ulysses_emulated(sp, Hq, Hkv):
    from tinytron_b200.ops import _ext, check_status
    from tinytron_b200.parallel.symm import SymmetricHeap
    from tinytron_b200.parallel.ulysses import kv_heads_for_rank

    C = _ext.load()
    B, T, D = 2, 64, 128
    hq_l = Hq // sp
    kv0 = [kv_heads_for_rank(r, sp, Hq, Hkv)[0] for r in range(sp)]
    hkv_l = kv_heads_for_rank(0, sp, Hq, Hkv)[1] - kv0[0]
    W = (hq_l + 2 * hkv_l) * D
    nbytes = sp * B * T * W * 2
    heaps = SymmetricHeap.create_emulated(2 * nbytes + 4096, sp)
    slots = [h.replay_slots(nbytes) for h in heaps]
    g = torch.Generator(device="cuda").manual_seed(sp * 10 + Hkv)
    qkvs = [torch.randn(B * T, (Hq + 2 * Hkv) * D, device="cuda", generator=g).bfloat16() for _ in range(sp)]

    def run_pack(src_list, rows, Wc, s1, s2, b0, b1, b2):
        for h, (buf, sb), src in zip(heaps, slots, src_list):
            C.ul_pack(h.gid, h.offset_of(buf), sb, src, B, T, rows, Wc, s1, s2, b0, b1, b2)

    # forward q|k|v -> heads, twice (the slots alternate through the device epoch)
    for _ in range(2):
        run_pack(qkvs, [T, 0, 1], W, hq_l * D, (hq_l + hkv_l) * D, [c * hq_l * D for c in range(sp)],
                 [Hq * D + k * D for k in kv0], [(Hq + Hkv) * D + k * D for k in kv0])
        fulls = [torch.empty(B * sp * T, W, device="cuda", dtype=torch.bfloat16) for _ in range(sp)]
        for h, (buf, sb), out in zip(heaps, slots, fulls):
            C.ul_exchange(h.gid, h.offset_of(buf), sb, out, B, T, [sp * T, T, 1], 0, W)
        torch.cuda.synchronize()
        check_status()
        for r in range(sp):
            assert torch.equal(fulls[r], _ref_full(qkvs, B, T, Hq, Hkv, D, sp, r)), r

    # backward: gradients of every rank's full buffer -> d(q|k|v) per rank (kv summed)
    gfulls = [torch.randn(B * sp * T, W, device="cuda", generator=g).bfloat16() for _ in range(sp)]
    run_pack(gfulls, [sp * T, T, 1], W, W, W, [0] * sp, [0] * sp, [0] * sp)
    dq = [torch.empty(B * T, (Hq + 2 * Hkv) * D, device="cuda", dtype=torch.bfloat16) for _ in range(sp)]
    for h, (buf, sb), out in zip(heaps, slots, dq):
        C.ul_exchange_qkv_grad(h.gid, h.offset_of(buf), sb, out, B, T, Hq, Hkv, D, hq_l, hkv_l, kv0)
    torch.cuda.synchronize()
    check_status()
    # reference: autograd through the plain-op construction
    leaves = [q.float().requires_grad_(True) for q in qkvs]
    tot = sum((_ref_full(leaves, B, T, Hq, Hkv, D, sp, r) * gfulls[r].float()).sum() for r in range(sp))
    tot.backward()
    for r in range(sp):
        assert ((dq[r].float() - leaves[r].grad).abs().max() / leaves[r].grad.abs().max()).item() < 1e-2, r

    # attention output direction: heads -> tokens and its backward
    Wo = hq_l * D
    os_ = [torch.randn(B * sp * T, Wo, device="cuda", generator=g).bfloat16() for _ in range(sp)]
    run_pack(os_, [sp * T, T, 1], Wo, Wo, Wo, [0] * sp, [0] * sp, [0] * sp)
    ys = [torch.empty(B * T, Hq * D, device="cuda", dtype=torch.bfloat16) for _ in range(sp)]
    for h, (buf, sb), out in zip(heaps, slots, ys):
        C.ul_exchange(h.gid, h.offset_of(buf), sb, out, B, T, [T, 0, 1], Wo, Wo)
    torch.cuda.synchronize()
    for r in range(sp):  # token chunk r, head block c from rank c
        want = torch.cat([os_[c].view(B, sp, T, Wo)[:, r] for c in range(sp)], -1).reshape(B * T, Hq * D)
        assert torch.equal(ys[r], want), r
    run_pack(ys, [T, 0, 1], Wo, Wo, Wo, [c * Wo for c in range(sp)], [0] * sp, [0] * sp)
    back = [torch.empty(B * sp * T, Wo, device="cuda", dtype=torch.bfloat16) for _ in range(sp)]
    for h, (buf, sb), out in zip(heaps, slots, back):
        C.ul_exchange(h.gid, h.offset_of(buf), sb, out, B, T, [sp * T, T, 1], 0, Wo)
    torch.cuda.synchronize()
    check_status()
    for r in range(sp):  # the round trip restores every rank's head-major buffer
        assert torch.equal(back[r], os_[r]), r
    for h in heaps:
        h.close()


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _cfg():
    from tinytron_b200.models import ModelConfig

    return ModelConfig(block_size=512, vocab_size=1024, num_layer=2, num_attention_heads=8, num_key_value_heads=2,
                       hidden_size=1024, intermediate_size=1024, init_std=0.02, seed=5)


def _data():
    g = torch.Generator().manual_seed(1)
    return torch.randint(0, 1024, (2, 512), generator=g), torch.randint(0, 1024, (2, 512), generator=g)


def _sep_worker(rank, world, port, q):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    try:
        from tinytron_b200.models import GPT
        from tinytron_b200.ops import check_status
        from tinytron_b200.parallel import parallel_state
        from tinytron_b200.parallel.buffers import FlatParams
        from tinytron_b200.parallel.symm import enable_heap_all_to_all
        from tinytron_b200.training.config import ParallelConfig

        parallel_state.initialize_model_parallel(ParallelConfig(sep_size=world))
        enable_heap_all_to_all(parallel_state.get_sp_group(), torch.device("cuda", rank))
        m = GPT(_cfg(), device=f"cuda:{rank}")
        flat = FlatParams(m)
        x, y = _data()
        T = x.shape[1] // world
        sl = slice(rank * T, (rank + 1) * T)
        _, loss, ll = m(x[:, sl].cuda(), y[:, sl].cuda())
        loss.backward()
        torch.cuda.synchronize()
        check_status()
        g = flat.grad[:flat.dense_numel].clone()
        dist.all_reduce(g, group=parallel_state.get_sp_group())  # SP sum of the dense grads
        q.put((rank, {"loss": float(ll), "grad": g.cpu()}))
        dist.barrier()
        parallel_state.destroy_model_parallel()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_two_rank_sep_attention_matches_single_rank():
    import torch.multiprocessing as mp

    from tinytron_b200.models import GPT
    from tinytron_b200.parallel.buffers import FlatParams

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_sep_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in range(2))
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    m = GPT(_cfg(), device="cuda:0")
    flat = FlatParams(m)
    x, y = _data()
    _, loss, ll = m(x.cuda(), y.cuda())
    loss.backward()
    assert abs(res[0]["loss"] - float(ll)) < 2e-2 and abs(res[1]["loss"] - float(ll)) < 2e-2
    ref = flat.grad[:flat.dense_numel].cpu()
    for r in range(2):
        assert ((res[r]["grad"] - ref).norm() / ref.norm()).item() < 5e-2, r
