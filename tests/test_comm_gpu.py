"""tt_comm symmetric-heap collectives vs plain PyTorch fp32 references.

Single GPU: W heaps on one device act as W ranks ("emulated" groups); each rank's
kernel is launched in turn with its peer waits disabled, so no kernel waits on
another.  The bounded-wait test launches ONE rank's barrier whose peer never
signals and checks that the wait gives up with a status code (the context stays
usable).  With two or more GPUs, a spawned 2-process NCCL group also checks the
real IPC-mapped path against NCCL.
"""
import math
import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _ref_adamw(p, g, m, v, lr, b1, b2, eps, wd, step):
    p = p * (1 - lr * wd)
    m = m + (1 - b1) * (g - m)
    v = b2 * v + (1 - b2) * g * g
    denom = v.sqrt() / math.sqrt(1 - b2 ** step) + eps
    return p - (lr / (1 - b1 ** step)) * (m / denom), m, v


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("W,n", [(2, 1000), (4, 4096 * 3 + 8), (8, 65536)])
def test_emulated_all_reduce(W, n, dtype):
    from tinytron_b200.parallel.symm import SymmetricHeap

    heaps = SymmetricHeap.create_emulated(2 * n * 4 + 4096, W)
    g = torch.Generator(device="cuda").manual_seed(W)
    srcs = []
    for h in heaps:
        t = h.alloc(n, dtype)
        t.copy_(torch.randn(n, device="cuda", generator=g).to(dtype))
        srcs.append(t)
    res = torch.randn(n, device="cuda", generator=g).to(dtype)
    ref = sum(s.float() for s in srcs) + res.float()
    outs = [h.all_reduce(s, residual=res) for h, s in zip(heaps, srcs)]
    torch.cuda.synchronize()
    tol = 2e-2 if dtype == torch.bfloat16 else 1e-5
    for o in outs:
        assert ((o.float() - ref).abs().max() / ref.abs().max()).item() < tol
        assert torch.equal(o, outs[0])  # same rank order everywhere: bit-identical
    for h in heaps:
        h.close()


@pytest.mark.parametrize("W", [2, 4, 8])
def test_emulated_zero1_step(W):
    """reduce-scatter + global-norm clip + AdamW + all-gather + shadow refresh on W
    emulated ranks == the fp32 reference update applied to the averaged gradient."""
    from tinytron_b200.parallel.symm import SymmetricHeap

    n = 64 * W * 37  # flat numel padded to a multiple of 64*W, as FlatParams does
    split = 64 * 11 * W  # dense / expert boundary (multiple of 64)
    shard = n // W
    lr, b1, b2, eps, wd, max_norm = 1e-2, 0.9, 0.95, 1e-8, 0.1, 0.5
    heaps = SymmetricHeap.create_emulated(SymmetricHeap.bytes_needed((n, torch.float32), (n, torch.float32),
                                                                     (n, torch.bfloat16)), W)
    g0 = torch.Generator(device="cuda").manual_seed(1)
    p0 = torch.randn(n, device="cuda", generator=g0)
    bufs = []
    for h in heaps:
        data, grad, p16 = h.alloc(n, torch.float32), h.alloc(n, torch.float32), h.alloc(n, torch.bfloat16)
        data.copy_(p0)
        p16.copy_(p0)
        bufs.append(dict(data=data, grad=grad, p16=p16, m=torch.zeros(shard, device="cuda"),
                         v=torch.zeros(shard, device="cuda"), norm=torch.zeros(2, device="cuda")))
    p_ref, m_ref, v_ref = p0.clone(), torch.zeros(n, device="cuda"), torch.zeros(n, device="cuda")
    for step in (1, 2):
        grads = [torch.randn(n, device="cuda", generator=g0) for _ in range(W)]
        for b, gr in zip(bufs, grads):
            b["grad"].copy_(gr)
        for r, (h, b) in enumerate(zip(heaps, bufs)):
            h.reduce_scatter_sumsq(b["grad"], r * shard, (r + 1) * shard, split, 1.0 / W)
        for r, (h, b) in enumerate(zip(heaps, bufs)):
            h.adamw_allgather(b["data"], b["grad"], b["p16"], b["m"], b["v"], r * shard, (r + 1) * shard, lr, (b1, b2),
                              eps, wd, step, max_norm, norm_out=b["norm"])
        for r, (h, b) in enumerate(zip(heaps, bufs)):
            h.shadow_refresh(b["data"], b["p16"], r * shard, (r + 1) * shard)
        torch.cuda.synchronize()
        gbar = torch.stack(grads).double().mean(0)
        norm = gbar.norm().item()
        coef = min(max_norm / (norm + 1e-6), 1.0)
        p_ref, m_ref, v_ref = _ref_adamw(p_ref.double(), gbar * coef, m_ref.double(), v_ref.double(), lr, b1, b2, eps,
                                         wd, step)
        for r, b in enumerate(bufs):
            assert abs(b["norm"][0].item() - norm) < 1e-4 * norm
            assert abs(b["norm"][1].item() - coef) < 1e-4
            assert (b["data"].double() - p_ref).abs().max().item() < 1e-5
            assert torch.equal(b["p16"], b["data"].bfloat16())
            sl = slice(r * shard, (r + 1) * shard)
            assert (b["m"].double() - m_ref[sl]).abs().max().item() < 1e-6
            assert (b["grad"][sl].double() - gbar[sl]).abs().max().item() < 1e-5
        for b in bufs[1:]:
            assert torch.equal(b["data"], bufs[0]["data"])
    for h in heaps:
        h.close()


@pytest.mark.parametrize("W,n", [(2, 8), (4, 1024), (8, 4096)])
def test_emulated_all_to_all(W, n):
    from tinytron_b200.parallel.symm import SymmetricHeap

    heaps = SymmetricHeap.create_emulated(W * n * 2 + 4096, W)
    slots = []
    for r, h in enumerate(heaps):
        s = h.alloc((W, n), torch.bfloat16)
        s.copy_(torch.arange(W * n, device="cuda").view(W, n).bfloat16() + 1000 * r)
        slots.append(s)
    outs = [h.all_to_all(s, torch.empty_like(s)) for h, s in zip(heaps, slots)]
    torch.cuda.synchronize()
    for me, o in enumerate(outs):
        for c in range(W):
            assert torch.equal(o[c], slots[c][me])
    for h in heaps:
        h.close()


def test_peer_wait_gives_up_with_status():
    """A barrier whose peer never signals returns after the (short) bound with
    kTimeoutPeer in the status word; the context stays usable afterwards."""
    from tinytron_b200.ops import _ext, check_status
    from tinytron_b200.parallel.symm import SymmetricHeap

    C = _ext.load()
    heaps = SymmetricHeap.create_emulated(4096, 2, waits=True)
    C.comm_set_timeout(0.5)
    try:
        heaps[0].barrier()  # rank 1 is never launched: nothing sets its flag
        torch.cuda.synchronize()
        code = int(C.status_read(torch.cuda.current_device()))
        assert code == 5, code
        C.status_clear(torch.cuda.current_device())
        check_status()
        x = torch.ones(4, device="cuda") * 2  # context still healthy
        assert x.sum().item() == 8
    finally:
        C.comm_set_timeout(60.0)
        for h in heaps:
            h.close()


# --------------------------------------------------------------------------- two real ranks
def _two_rank_worker(rank, world, port, out_q):
    import torch.distributed as dist

    from tinytron_b200.parallel.symm import SymmetricHeap

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    try:
        n = 64 * world * 1000
        shard = n // world
        heap = SymmetricHeap.create(SymmetricHeap.bytes_needed((n, torch.float32), (n, torch.float32),
                                                               (n, torch.bfloat16), (n, torch.bfloat16)))
        g = torch.Generator(device="cuda").manual_seed(100 + rank)
        src = heap.alloc(n, torch.bfloat16)
        src.copy_(torch.randn(n, device="cuda", generator=g).bfloat16())
        ours = heap.all_reduce(src)
        ref = src.float().clone()
        dist.all_reduce(ref)
        ar_err = ((ours.float() - ref).abs().max() / ref.abs().max()).item()
        # ZeRO-1 step vs NCCL reduce-scatter + reference AdamW + all-gather
        data, grad = heap.alloc(n, torch.float32), heap.alloc(n, torch.float32)
        p16 = heap.alloc(n, torch.bfloat16)
        torch.manual_seed(0)
        p0 = torch.randn(n, device="cuda")
        data.copy_(p0)
        p16.copy_(p0)
        gr = torch.randn(n, device="cuda", generator=g)
        grad.copy_(gr)
        m, v, nrm = torch.zeros(shard, device="cuda"), torch.zeros(shard, device="cuda"), torch.zeros(2, device="cuda")
        lo, hi = rank * shard, (rank + 1) * shard
        heap.reduce_scatter_sumsq(grad, lo, hi, n, 1.0 / world)
        heap.adamw_allgather(data, grad, p16, m, v, lo, hi, 1e-2, (0.9, 0.95), 1e-8, 0.1, 1, 1.0, norm_out=nrm)
        heap.shadow_refresh(data, p16, lo, hi)
        gsum = gr.clone()
        dist.all_reduce(gsum)
        gbar = gsum / world
        coef = min(1.0 / (gbar.norm().item() + 1e-6), 1.0)
        pr, _, _ = _ref_adamw(p0, gbar * coef, torch.zeros_like(p0), torch.zeros_like(p0), 1e-2, 0.9, 0.95, 1e-8, 0.1,
                              1)
        z_err = (data - pr).abs().max().item()
        from tinytron_b200.parallel.symm import HeapAllToAll

        a2a = HeapAllToAll(None)
        x = torch.randn(world, 3, 64, device="cuda", generator=g).bfloat16()
        slot = a2a.slot(x.shape, x.dtype)
        slot.copy_(x)
        ours_a2a = a2a.exchange(slot)
        ref_a2a = torch.empty_like(x)
        dist.all_to_all_single(ref_a2a, x.contiguous())
        z_err = max(z_err, (ours_a2a.float() - ref_a2a.float()).abs().max().item())
        shadow_ok = bool(torch.equal(p16, data.bfloat16()))
        torch.cuda.synchronize()
        from tinytron_b200.ops import check_status

        check_status()
        dist.barrier()
        heap.close()
        out_q.put((rank, ar_err, z_err, shadow_ok))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_two_rank_ipc_collectives_match_nccl():
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_two_rank_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    res = sorted(q.get(timeout=5) for _ in range(2))
    for rank, ar_err, z_err, shadow_ok in res:
        assert ar_err < 2e-2, (rank, ar_err)
        assert z_err < 1e-5, (rank, z_err)
        assert shadow_ok, rank


@pytest.mark.parametrize("W", [2, 4, 8])
def test_emulated_bucketed_zero1_step(W):
    """The overlapped-reduce-scatter layout: buckets of the flat buffer, rank r owning the
    r-th slice of every bucket (reduce per bucket with the sums of squares kept local, one
    publish, AdamW per slice, full shadow refresh) == the fp32 reference update."""
    from tinytron_b200.parallel.symm import SymmetricHeap

    n = 64 * W * 37
    split = 64 * 11 * W
    bounds = [0, 64 * W * 5, 64 * W * 20, n]  # three buckets
    buckets = list(zip(bounds[:-1], bounds[1:]))
    lr, b1, b2, eps, wd, max_norm = 1e-2, 0.9, 0.95, 1e-8, 0.1, 0.5
    heaps = SymmetricHeap.create_emulated(SymmetricHeap.bytes_needed((n, torch.float32), (n, torch.float32),
                                                                     (n, torch.bfloat16)), W)
    g0 = torch.Generator(device="cuda").manual_seed(2)
    p0 = torch.randn(n, device="cuda", generator=g0)
    bufs = []
    for h in heaps:
        data, grad, p16 = h.alloc(n, torch.float32), h.alloc(n, torch.float32), h.alloc(n, torch.bfloat16)
        data.copy_(p0)
        p16.copy_(p0)
        bufs.append(dict(data=data, grad=grad, p16=p16, m=torch.zeros(n // W, device="cuda"),
                         v=torch.zeros(n // W, device="cuda"), norm=torch.zeros(2, device="cuda"),
                         sq=torch.zeros(len(buckets), 2, device="cuda")))

    def my_slices(r):
        out, off = [], 0
        for lo, hi in buckets:
            k = (hi - lo) // W
            out.append(((lo + r * k, lo + (r + 1) * k), (off, off + k)))
            off += k
        return out

    p_ref, m_ref, v_ref = p0.clone().double(), torch.zeros(n, device="cuda").double(), torch.zeros(n, device="cuda").double()
    for step in (1, 2):
        grads = [torch.randn(n, device="cuda", generator=g0) for _ in range(W)]
        for b, gr in zip(bufs, grads):
            b["grad"].copy_(gr)
        for bi in range(len(buckets)):  # bucket by bucket, every rank (launch order = overlap order)
            for r, (h, b) in enumerate(zip(heaps, bufs)):
                (lo, hi), _ = my_slices(r)[bi]
                h.reduce_scatter_bucket(b["grad"], lo, hi, split, 1.0 / W, b["sq"][bi])
        pads = [h.publish_sumsq(b["sq"]) for h, b in zip(heaps, bufs)]
        for r, (h, b) in enumerate(zip(heaps, bufs)):
            for (lo, hi), (m0, m1) in my_slices(r):
                h.adamw_allgather(b["data"], b["grad"], b["p16"], b["m"][m0:m1], b["v"][m0:m1], lo, hi, lr, (b1, b2),
                                  eps, wd, step, max_norm, norm_out=b["norm"], pads_epoch=pads[r])
        for h, b in zip(heaps, bufs):
            h.shadow_refresh(b["data"], b["p16"], 0, 0)
        torch.cuda.synchronize()
        gbar = torch.stack(grads).double().mean(0)
        norm = gbar.norm().item()
        coef = min(max_norm / (norm + 1e-6), 1.0)
        p_ref, m_ref, v_ref = _ref_adamw(p_ref, gbar * coef, m_ref, v_ref, lr, b1, b2, eps, wd, step)
        for b in bufs:
            assert abs(b["norm"][0].item() - norm) < 1e-4 * norm
            # fp32 AdamW against the fp64 reference: elements whose gradient is near eps
            # differ by a few 1e-5 after two steps; a wrong slice or state offset is O(lr)
            assert (b["data"].double() - p_ref).abs().max().item() < 5e-5
            assert torch.equal(b["p16"], b["data"].bfloat16())
        for b in bufs[1:]:
            assert torch.equal(b["data"], bufs[0]["data"])  # every rank holds the same parameters
    for h in heaps:
        h.close()
