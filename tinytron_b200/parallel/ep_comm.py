"""Expert parallelism over NVLink peer memory (Python side of ``csrc/moe/ep.cu``).

Replaces the reference's EP path (``tinytron/model/modules/mlp.py:257-293`` and
``tinytron/distributed/expert_parallel/comm.py:22-164``: sort by target rank, count
all-to-all + ``.cpu().tolist()``, padded variable all-to-alls of hidden rows and
expert ids, local sort, grouped GEMM, reverse all-to-all, unsort, weighted sum).

Here, per MoE layer and micro-step:

1. routing metadata on the device (per-expert counts, each pair's rank within its
   expert); one small kernel all-gathers the [E] count vectors into a [world, E]
   matrix in every rank's heap; the host reads that matrix (the only host sync,
   64 x world ints) and computes every rank's 128- or 256-row-aligned expert segments, so
   each (token, slot) pair knows its destination row in the owner's buffer;
2. ``ep_scatter``: a warp per pair stores the token row straight into the owner's
   expert-grouped receive buffer (no send-side sort copy, no all-to-all);
3. the owner runs its local experts on the grouped tcgen05 GEMMs (gate|up with the
   SwiGLU epilogue, then down).  With ``TT_EP_PUSH_COMBINE=1`` the combine
   all-to-all is fused into the down projection: the scatter of step 2 also recorded,
   per received row, the sender's rank and the slot of that (token, slot) pair in the
   sender's return buffer; ``ep_resolve_rows`` turns the records into peer addresses
   and the GEMM's epilogue stores each output row straight into the sender's memory,
   so the NVLink transfer overlaps the GEMM tile by tile;
4. a barrier, then the routing-weighted sum of each token's k rows: loaded from the
   owners' output buffers (``ep_pull_combine``, peer loads; the default) or, in push
   mode, from the local return buffer (``ep_local_combine``).  Pull is the default
   because it measured faster: at SEP=2 the push epilogue's per-row peer stores made the
   down projection 3.3x slower (61 vs 18 ms per step) while the pull-combine costs 17 ms
   more, 557 vs 584 ms per step in all.

The backward mirrors it: ``ep_scatter`` in backward mode sends w * dout rows (and
computes d(weights) on the way), the owner runs the expert backward into its output
buffer, and the pull-combine sums the k input-gradient rows per token.

Buffer reuse across layers is safe without extra barriers: a rank writes a peer's
receive buffer for layer l+1 only after that peer passed layer l's output barrier
(so its GEMMs have read the buffer), and an owner writes its output buffer for l+1
only after every source scattered l+1, i.e. finished pulling l.
"""
from __future__ import annotations

import os

import numpy as np
import torch
import torch.distributed as dist

from tinytron_b200.ops.weights import bf16_of, concat_rows_cached, main_grad_of, notify_grad_ready

from .symm import SymmetricHeap

ALIGN_ROWS = 256  # largest segment alignment (capacity bound); see plan_finish


def _C():
    from tinytron_b200.ops import _ext

    return _ext.load()


def push_combine_enabled() -> bool:
    """Combine fused into the down-projection epilogue (peer stores); off (default): pull-combine."""
    return os.environ.get("TT_EP_PUSH_COMBINE", "0") == "1"


class EPBuffers:
    """Per-EP-group symmetric heap: a [world, E] count matrix, two [cap, H] bf16 row
    buffers (A: receive rows / incoming gradients, B: expert outputs -- in push mode the
    return rows of this rank's own pairs -- / input gradients) and a [cap] int64 array of
    return-address records (push mode)."""

    def __init__(self, heap: SymmetricHeap, E: int, H: int, cap: int):
        self.heap = heap
        self.world, self.rank = heap.world, heap.rank
        self.E, self.H, self.cap = E, H, cap
        self.counts = heap.alloc((self.world, E), torch.int32)
        self.buf_a = heap.alloc((cap, H), torch.bfloat16, zero=False)
        self.buf_b = heap.alloc((cap, H), torch.bfloat16, zero=False)
        self.ret = heap.alloc(cap, torch.int64)  # zero = no record
        self.off_counts = heap.offset_of(self.counts)
        self.off_a = heap.offset_of(self.buf_a)
        self.off_b = heap.offset_of(self.buf_b)
        self.off_ret = heap.offset_of(self.ret)

    @staticmethod
    def nbytes(world: int, E: int, H: int, cap: int) -> int:
        return SymmetricHeap.bytes_needed((world * E, torch.int32), (cap * H, torch.bfloat16),
                                          (cap * H, torch.bfloat16), (cap, torch.int64))

    @classmethod
    def create(cls, group, E: int, H: int, cap: int, device=None) -> "EPBuffers":
        world = dist.get_world_size(group)
        return cls(SymmetricHeap.create(cls.nbytes(world, E, H, cap), group, device), E, H, cap)

    @classmethod
    def create_emulated(cls, world: int, E: int, H: int, cap: int, device=None) -> list["EPBuffers"]:
        heaps = SymmetricHeap.create_emulated(cls.nbytes(world, E, H, cap), world, device)
        return [cls(h, E, H, cap) for h in heaps]

    def close(self):
        self.heap.close()


def capacity(world: int, tokens: int, k: int, local_experts: int) -> int:
    """Worst-case receive rows: every pair of every rank routed here, plus segment padding."""
    return world * tokens * k + local_experts * ALIGN_ROWS


_BUFFERS: dict = {}


def get_ep_buffers(group, E: int, H: int, tokens: int, k: int, device=None) -> EPBuffers:
    """Collective over ``group`` on first use (or when a larger capacity is needed)."""
    world = dist.get_world_size(group)
    cap = capacity(world, tokens, k, E // world)
    key = id(group)
    b = _BUFFERS.get(key)
    if b is None or b.cap < cap or b.E != E or b.H != H:
        if b is not None:
            b.close()
        b = EPBuffers.create(group, E, H, cap, device)
        _BUFFERS[key] = b
    return b


# ---------------------------------------------------------------------------- phases
class Plan:
    """Where every (token, slot) pair of this rank goes, and this rank's receive layout."""

    __slots__ = ("tgt", "dst", "grp_off", "seg_cnt", "total", "k", "N", "E_local", "pair")


def plan_routes(bufs: EPBuffers, sel: torch.Tensor) -> torch.Tensor:
    """Phase 1a (collective): publish this rank's per-expert counts; returns them."""
    flat = sel.reshape(-1).long()
    counts = torch.bincount(flat, minlength=bufs.E).to(torch.int32)
    _C().ep_allgather_counts(bufs.heap.gid, counts, bufs.off_counts)
    return counts


def plan_finish(bufs: EPBuffers, sel: torch.Tensor, counts: torch.Tensor, M: np.ndarray | None = None) -> Plan:
    """Phase 1b (local): destination rows of this rank's pairs and its receive segments.
    ``M`` ([world, E] counts of every rank) is read from the heap unless given."""
    world, rank, E = bufs.world, bufs.rank, bufs.E
    E_l = E // world
    N, k = sel.shape
    if M is None:
        M = bufs.counts.cpu().numpy().astype(np.int64)  # host sync: world x E ints
    n = M.sum(0).reshape(world, E_l)  # rows each owner receives per local expert
    # 256-row segments (CTA-pair grouped GEMMs) when experts average >= 256 rows, else 128
    align = 256 if int(M.sum()) >= 256 * E else 128
    seg = (n + align - 1) // align * align
    seg_off = np.cumsum(seg, axis=1) - seg  # [world, E_l] segment starts in each owner's buffer
    src_before = np.cumsum(M, axis=0) - M  # [world(src), E] rows of earlier sources
    base = seg_off.reshape(E) + src_before[rank]  # [E] first row of this rank's pairs per expert
    total = int(seg[rank].sum())
    if int(seg.sum(1).max()) > bufs.cap:
        raise RuntimeError(f"EP receive buffer too small ({int(seg.sum(1).max())} > {bufs.cap} rows)")
    dev = sel.device
    p = Plan()
    p.total, p.k, p.N, p.E_local = total, k, N, E_l
    p.pair = align == 256
    if sel.is_cuda:
        # stable position of every pair within its expert from the layout kernel (unpadded
        # segments), then one kernel for dst/tgt; the per-expert offsets and the receive
        # segments travel to the device in one copy
        c = _C()
        sel32 = sel.reshape(-1).to(torch.int32).contiguous()
        P = sel32.numel()
        lay = torch.empty(E + 1, dtype=torch.int32, device=dev)
        slot = torch.empty(P, dtype=torch.int32, device=dev)
        rows = torch.empty(max(P, 1), dtype=torch.int32, device=dev)
        c.moe_layout(sel32, E, lay, slot, rows, 1)
        mine = M[rank]
        start = np.cumsum(mine) - mine  # first position of each expert in the sorted order
        meta = np.concatenate([base - start, seg_off[rank], [total], n[rank]]).astype(np.int32)
        meta = torch.from_numpy(meta).pin_memory().to(dev, non_blocking=True)
        p.grp_off, p.seg_cnt = meta[E:E + E_l + 1], meta[E + E_l + 1:]
        p.dst = torch.empty(P, dtype=torch.int32, device=dev)
        p.tgt = torch.empty(P, dtype=torch.int32, device=dev)
        c.ep_plan_rows(sel32, slot, meta[:E], E_l, p.dst, p.tgt)
        return p
    flat = sel.reshape(-1).long()
    P = flat.numel()
    order = torch.argsort(flat, stable=True)
    start = torch.cumsum(counts.long(), 0) - counts.long()
    rank_in_e = torch.empty(P, dtype=torch.long, device=dev)
    rank_in_e[order] = torch.arange(P, device=dev) - start[flat[order]]
    p.dst = (torch.from_numpy(base).to(dev)[flat] + rank_in_e).to(torch.int32).contiguous()
    p.tgt = (flat // E_l).to(torch.int32).contiguous()
    p.grp_off = torch.tensor(list(seg_off[rank]) + [total], dtype=torch.int32, device=dev)
    p.seg_cnt = torch.tensor(n[rank], dtype=torch.int32, device=dev)
    return p


def dispatch(bufs: EPBuffers, plan: Plan, x2d: torch.Tensor, push: bool = False) -> torch.Tensor:
    """Phase 2 (collective): rows to owners; returns this rank's grouped receive rows.
    ``push``: also record each row's return slot (this rank, pair index) at the owner."""
    C = _C()
    if push:
        C.ep_scatter(bufs.heap.gid, x2d, plan.k, plan.tgt, plan.dst, bufs.off_a, bufs.cap, None, None, None,
                     bufs.off_ret, bufs.off_b)
    else:
        C.ep_scatter(bufs.heap.gid, x2d, plan.k, plan.tgt, plan.dst, bufs.off_a, bufs.cap, None, None, None)
    xr = bufs.buf_a[:plan.total]
    C.ep_zero_pad(xr, plan.grp_off, plan.seg_cnt)
    return xr


def experts_forward(bufs: EPBuffers, plan: Plan, xr: torch.Tensor, w_gu: torch.Tensor, wd: torch.Tensor, I: int,
                    push: bool = False):
    """Phase 3 (local): grouped SwiGLU experts; outputs land in buffer B (pull mode) or,
    ``push``, in the senders' return buffers straight from the down-projection epilogue."""
    C = _C()
    dev = xr.device
    act = torch.empty(plan.total, I, device=dev, dtype=torch.bfloat16)
    gu = torch.empty(plan.total, 2 * I, device=dev, dtype=torch.bfloat16)
    yr = bufs.buf_b[:plan.total]
    row_ptr = None
    if push:
        row_ptr = torch.empty(max(plan.total, 1), device=dev, dtype=torch.int64)
        C.ep_resolve_rows(bufs.heap.gid, bufs.off_ret, plan.total, bufs.H, row_ptr)
    if plan.total > 0:
        C.moe_gemm_swiglu(xr, w_gu, act, gu, plan.grp_off, plan.E_local, plan.pair)
        # push mode: `yr` only gives the output shape; rows go to row_ptr[r]
        C.moe_gemm(act, wd, yr, plan.grp_off, plan.E_local, False, bufs.H, 0, 0, plan.pair, row_ptr)
    return act, gu


def combine(bufs: EPBuffers, plan: Plan, w32: torch.Tensor | None, keep_rows: bool, push: bool = False):
    """Phase 4 (collective): barrier, then the weighted sum of each token's k rows (read
    from the owners, or from this rank's return buffer after a pushed exchange)."""
    C = _C()
    bufs.heap.barrier()
    dev = plan.tgt.device
    out = torch.empty(plan.N, bufs.H, device=dev, dtype=torch.bfloat16)
    rows = torch.empty(plan.N * plan.k, bufs.H, device=dev, dtype=torch.bfloat16) if keep_rows else None
    if push:
        C.ep_local_combine(bufs.heap.gid, bufs.off_b, plan.k, w32, out, rows)
    else:
        C.ep_pull_combine(bufs.heap.gid, bufs.off_b, bufs.cap, plan.tgt, plan.dst, plan.k, w32, out, rows)
    return out, rows


def grad_dispatch(bufs: EPBuffers, plan: Plan, d2d: torch.Tensor, w32: torch.Tensor, rows: torch.Tensor):
    """Backward phase 1 (collective): w * dout rows to the owners; d(weights) on the way."""
    C = _C()
    dw = torch.empty(plan.N * plan.k, device=d2d.device, dtype=torch.float32)
    C.ep_scatter(bufs.heap.gid, d2d, plan.k, plan.tgt, plan.dst, bufs.off_a, bufs.cap, w32, rows, dw)
    dyr = bufs.buf_a[:plan.total]
    C.ep_zero_pad(dyr, plan.grp_off, plan.seg_cnt)
    return dyr, dw


def experts_backward(bufs: EPBuffers, plan: Plan, dyr, xr, act, gu, w_gu, wd, I, g_gate, g_up, g_down) -> None:
    """Backward phase 2 (local): SwiGLU + down backward on the grouped GEMMs, weight
    gradients accumulated into g_*, input gradients into buffer B."""
    if plan.total == 0:
        return
    C = _C()
    E_l = plan.E_local
    dgu = torch.empty(plan.total, 2 * I, device=dyr.device, dtype=torch.bfloat16)
    C.moe_gemm_dswiglu(dyr, wd, gu, dgu, plan.grp_off, E_l, plan.pair)
    C.moe_gemm_wgrad(dyr, act, g_down, plan.grp_off, E_l, True, True)
    C.moe_gemm(dgu, w_gu, bufs.buf_b[:plan.total], plan.grp_off, E_l, True, I, I, E_l * I, plan.pair)
    C.moe_gemm_wgrad(dgu[:, :I], xr, g_gate, plan.grp_off, E_l, True, True)
    C.moe_gemm_wgrad(dgu[:, I:], xr, g_up, plan.grp_off, E_l, True, True)


def _expert_grad(param, shape2d):
    mg = main_grad_of(param)
    if mg is not None:
        return mg.view(shape2d), True
    return torch.zeros(shape2d, device=param.device, dtype=torch.float32), False


class EPMoEFn(torch.autograd.Function):
    """Routed SwiGLU experts sharded over an EP group, dispatch/combine by peer stores
    and loads (see the module docstring).  x [N, H]; sel [N, k] global expert ids;
    weights [N, k] fp32 routing weights; expert weights are this rank's local experts."""

    @staticmethod
    def forward(ctx, x, sel, weights, w_gate, w_up, w_down, bufs):
        shape = x.shape
        x2d = x.reshape(-1, shape[-1]).to(torch.bfloat16).contiguous()
        E_l, I, H = w_gate.shape[0], w_gate.shape[1], w_gate.shape[2]
        counts = plan_routes(bufs, sel)
        plan = plan_finish(bufs, sel, counts)
        push = push_combine_enabled()
        xr = dispatch(bufs, plan, x2d, push)
        w_gu = concat_rows_cached(w_gate, "_tt_gu_cat", [bf16_of(w_gate).view(E_l * I, H), bf16_of(w_up).view(E_l * I, H)])
        wd = bf16_of(w_down).view(E_l * H, I)
        act, gu = experts_forward(bufs, plan, xr, w_gu, wd, I, push)
        w32 = weights.reshape(-1).float().contiguous()
        out, rows = combine(bufs, plan, w32, keep_rows=True, push=push)
        ctx.save_for_backward(xr.clone(), act, gu, rows, w32, w_gu, wd)
        ctx.plan, ctx.bufs, ctx.dims = plan, bufs, (E_l, I, H)
        ctx.params = (w_gate, w_up, w_down)
        ctx.shape = shape
        return out.view(shape)

    @staticmethod
    def backward(ctx, dout):
        xr, act, gu, rows, w32, w_gu, wd = ctx.saved_tensors
        plan, bufs = ctx.plan, ctx.bufs
        E_l, I, H = ctx.dims
        w_gate, w_up, w_down = ctx.params
        d2d = dout.reshape(-1, H).to(torch.bfloat16).contiguous()
        dyr, dw = grad_dispatch(bufs, plan, d2d, w32, rows)
        g_down, main_d = _expert_grad(w_down, (E_l * H, I))
        g_gate, main_g = _expert_grad(w_gate, (E_l * I, H))
        g_up, main_u = _expert_grad(w_up, (E_l * I, H))
        experts_backward(bufs, plan, dyr, xr, act, gu, w_gu, wd, I, g_gate, g_up, g_down)
        dx, _ = combine(bufs, plan, None, keep_rows=False)
        notify_grad_ready([p for p, m in ((w_gate, main_g), (w_up, main_u), (w_down, main_d)) if m])
        return (dx.view(ctx.shape), None, dw.view(plan.N, plan.k),
                None if main_g else g_gate.view_as(w_gate), None if main_u else g_up.view_as(w_up),
                None if main_d else g_down.view_as(w_down), None)


def ep_moe(x, sel, weights, w_gate, w_up, w_down, group):
    """y[t] = sum_j weights[t, j] * SwiGLU_{sel[t, j]}(x[t]) with experts sharded over ``group``."""
    N = x.reshape(-1, x.shape[-1]).shape[0]
    bufs = get_ep_buffers(group, w_gate.shape[0] * dist.get_world_size(group), x.shape[-1], N, sel.shape[-1],
                          x.device)
    return EPMoEFn.apply(x, sel.to(torch.int32), weights, w_gate, w_up, w_down, bufs)
