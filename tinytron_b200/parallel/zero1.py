"""ZeRO-1 optimizer-state sharding.

Two implementations:

* :class:`DistributedOptimizer` / :func:`partition_tensors` — API-compatible with the
  reference (tinytron/distributed/zero1/distributed_optimizer.py:6-185): wraps any
  torch optimizer, assigns whole tensors to DP ranks with a deterministic
  largest-first (LPT) greedy partition, steps only owned tensors and broadcasts
  them from their owners.  Used for Muon (whole matrices must live on one rank)
  and for user-supplied optimizers.

* :class:`FlatZeRO1` — the fast path for AdamW on :class:`FlatParams`: gradients are
  SP-summed (non-expert prefix) and DP reduce-scattered into equal contiguous
  shards, the global norm is one fused reduction plus a 2-float all-reduce, one
  fused kernel applies clip + AdamW to the owned shard (also writing the bf16
  shadow), and the updated master shard is all-gathered.  AdamW is elementwise,
  so element-wise sharding gives exactly the same update as whole-tensor sharding.

  When the flat buffers live in a symmetric heap (``FlatParams(heap_factory=...)``,
  one node, no SP expert split) the DP path runs on NVLink peer memory instead of
  NCCL: one kernel reduce-scatters the fp32 gradients by peer loads and publishes
  this rank's sums of squares into every peer's pad; a second kernel forms the clip
  coefficient from the pads, applies AdamW to the owned shard and stores the new
  fp32 shard straight into every peer's parameter buffer; a third waits for the
  peers' stores and refreshes the local bf16 shadow of their shards.

  With ``bucket_bytes`` (``--grad_bucket_mb``, DP only) the reduce-scatter overlaps the
  last micro-step's backward: the buffer is cut into buckets of whole parameters in
  reverse order, every rank owns one slice of every bucket, and each bucket's
  reduce-scatter kernel starts on a side stream (a few CTAs, next to the GEMMs) as soon
  as the wgrad epilogues of its last parameter have run.
"""
from __future__ import annotations

import heapq
import math
from collections import OrderedDict

import torch
import torch.distributed as dist


# ============================================================================ reference-compatible
class DistributedOptimizer:
    def __init__(self, optimizer, process_group, ranks_map=None, num_parts=None, verbose=False):
        object.__setattr__(self, "optimizer", optimizer)
        object.__setattr__(self, "process_group", process_group)
        object.__setattr__(self, "ranks_map", ranks_map)
        object.__setattr__(self, "num_parts", num_parts)
        object.__setattr__(self, "verbose", verbose)
        self.rank = dist.get_rank(process_group)
        self.world_size = dist.get_world_size(process_group)
        if self.num_parts is None:
            self.num_parts = self.world_size
        assert 1 <= self.num_parts <= self.world_size
        self.apply_zero1()

    def apply_zero1(self, part_assignment=None):
        self.tensor_dict = OrderedDict()
        for gi, group in enumerate(self.optimizer.param_groups):
            for pi, p in enumerate(group["params"]):
                if isinstance(p, torch.Tensor) and p.requires_grad:
                    self.tensor_dict[(gi, pi)] = p
        if part_assignment is None:
            if self.ranks_map is None:
                owners = list(range(self.num_parts))
            else:
                owners = [dist.get_group_rank(self.process_group, r) for r in self.ranks_map]
                self.num_parts = len(owners)
            assert len(set(owners)) == len(owners), f"Duplicate owners in ranks_map: {self.ranks_map}"
            part_assignment, _ = partition_tensors(self.tensor_dict, ranks_map=owners, num_parts=self.num_parts,
                                                   verbose=self.verbose)
        self.part_assignment = part_assignment
        for gi, group in enumerate(self.optimizer.param_groups):
            group["params"] = [p for pi, p in enumerate(group["params"])
                               if isinstance(p, torch.Tensor) and p.requires_grad
                               and self.part_assignment[(gi, pi)] == self.rank]
        dist.barrier(self.process_group)

    def __getattr__(self, name):
        return getattr(self.optimizer, name)

    def __setattr__(self, name, value):
        if name in {"optimizer", "process_group", "ranks_map", "num_parts", "verbose", "part_assignment",
                    "tensor_dict", "rank", "world_size"} or name.startswith("_"):
            object.__setattr__(self, name, value)
        else:
            setattr(self.optimizer, name, value)

    @torch.no_grad()
    def step(self, *args, **kwargs):
        out = self.optimizer.step(*args, **kwargs)
        if self.world_size > 1:
            self._broadcast_all_params_from_owners()
        return out

    @torch.no_grad()
    def zero_grad(self, set_to_none: bool = True):
        for p in self.tensor_dict.values():
            if p.grad is not None:
                if set_to_none:
                    p.grad = None
                else:
                    p.grad.zero_()

    @torch.no_grad()
    def _broadcast_all_params_from_owners(self):
        for key, p in self.tensor_dict.items():
            src = dist.get_global_rank(self.process_group, self.part_assignment[key])
            dist.broadcast(p.data, src=src, group=self.process_group)


def partition_tensors(tensor_dict, ranks_map=None, num_parts=None, verbose=False, deterministic=True):
    """Greedy largest-first assignment of tensors to parts (min-heap on load)."""
    if ranks_map is not None:
        num_parts = len(ranks_map)
    assert num_parts and num_parts > 0, "num_parts must be positive integer"
    items = [(k, t.numel()) for k, t in tensor_dict.items()]
    items.sort(key=(lambda x: (-x[1], x[0])) if deterministic else (lambda x: -x[1]))
    heap = [(0, i) for i in range(num_parts)]
    heapq.heapify(heap)
    assignment = {k: None for k in tensor_dict}
    sizes = {i: 0 for i in range(num_parts)}
    for key, size in items:
        cur, part = heapq.heappop(heap)
        assignment[key] = ranks_map[part] if ranks_map is not None else part
        sizes[part] = cur + size
        heapq.heappush(heap, (cur + size, part))
    if verbose:
        total = sum(sizes.values())
        imb = (max(sizes.values()) - min(sizes.values())) / (total / num_parts + 1e-6)
        print(f"[ZeRO-1] Partition load imbalance: {imb:.2%}")
    return assignment, tensor_dict


# ============================================================================ fast flat path
def plan_grad_buckets(offsets, numel: int, bucket_bytes: int, dp: int, dp_rank: int):
    """Buckets of whole parameters for the overlapped reduce-scatter, in REVERSE buffer
    order (the order gradients become final), each at least ``bucket_bytes`` of fp32
    gradients except possibly the last; they tile [0, numel).  Returns (buckets,
    this rank's slice of each bucket, the slice's offsets in the rank's optimizer state).
    Every bucket length is a multiple of 4 * dp (parameter offsets are multiples of 64
    and dp divides 16), so every slice is float4-aligned."""
    bounds = [numel]
    for o in sorted(offsets, reverse=True):
        if o > 0 and (bounds[-1] - o) * 4 >= bucket_bytes:
            bounds.append(o)
    if bounds[-1] != 0:
        bounds.append(0)
    buckets = [(bounds[i + 1], bounds[i]) for i in range(len(bounds) - 1)]
    slices, state_off, off = [], [], 0
    for lo, hi in buckets:
        if (hi - lo) % (4 * dp):
            raise ValueError(f"bucket [{lo}, {hi}) cannot be split into {dp} float4-aligned slices")
        n = (hi - lo) // dp
        slices.append((lo + dp_rank * n, lo + (dp_rank + 1) * n))
        state_off.append((off, off + n))
        off += n
    return buckets, slices, state_off


class FlatZeRO1:
    """Gradient sync + clip + fused AdamW + parameter all-gather over FlatParams.

    ``dp_group``/``sp_group`` may be None (size 1).  Semantics match the reference:
    non-expert grads SUM over SP, all grads AVG over DP (DDP), global-norm clip
    with expert norm^2 summed over EP, AdamW with decoupled weight decay on all
    parameters."""

    def __init__(self, flat, dp_group=None, sp_group=None, lr=1e-3, betas=(0.9, 0.95), eps=1e-8,
                 weight_decay=0.0, bucket_bytes: int = 0):
        self.flat = flat
        self.dp_group = dp_group
        self.sp_group = sp_group
        self.dp = dist.get_world_size(dp_group) if dp_group is not None else 1
        self.dp_rank = dist.get_rank(dp_group) if dp_group is not None else 0
        self.sp = dist.get_world_size(sp_group) if sp_group is not None else 1
        assert flat.numel % self.dp == 0, "flat buffer must be padded to a multiple of the DP size"
        self.shard = flat.numel // self.dp
        self.lo = self.dp_rank * self.shard
        self.hi = self.lo + self.shard
        self.param_groups = [{"lr": lr, "betas": betas, "eps": eps, "weight_decay": weight_decay}]
        dev = flat.device
        self.exp_avg = torch.zeros(self.shard, device=dev)
        self.exp_avg_sq = torch.zeros(self.shard, device=dev)
        self.step_count = 0
        self._scratch = torch.empty(4096, device=dev)
        self._sq = torch.zeros(2, device=dev)
        self._norm = torch.zeros(1, device=dev)
        self._coef = torch.ones(1, device=dev)
        self.master_synced = True
        heap = getattr(flat, "heap", None)
        # Native NVLink path: heap spans exactly this DP group and no SP-summed expert
        # norm term is needed (that one still takes the NCCL path).
        self.native = (heap is not None and self.dp > 1 and heap.world == self.dp
                       and (self.sp == 1 or flat.dense_numel == flat.numel) and self.shard % 4 == 0)
        self._max_norm = 0.0
        self._normc = torch.zeros(2, device=dev)
        self.buckets = None
        if self.native and bucket_bytes > 0 and self.sp == 1 and 16 % self.dp == 0 and dev.type == "cuda":
            self._init_buckets(int(bucket_bytes))

    # ---------------------------------------------------------------- overlapped reduce-scatter
    def _init_buckets(self, bucket_bytes: int) -> None:
        """Buckets of whole parameters in reverse buffer order (the order their gradients
        become final in the backward).  Ownership is interleaved: rank r owns the r-th of
        ``dp`` equal slices of EVERY bucket, so each bucket's reduce-scatter spreads over all
        ranks and can start as soon as that bucket is final everywhere."""
        flat = self.flat
        self.buckets, self.slices, self.state_off = plan_grad_buckets(flat.offsets, flat.numel, bucket_bytes,
                                                                      self.dp, self.dp_rank)
        assert self.state_off[-1][1] == self.shard
        self._bucket_of = {}
        self._bucket_params = [[] for _ in self.buckets]
        for p, o in zip(flat.params, flat.offsets):
            b = next(i for i, (lo, hi) in enumerate(self.buckets) if lo <= o < hi)
            self._bucket_of[id(p)] = b
            self._bucket_params[b].append(p)
        self._expected = None     # notifications per parameter in one micro-step (learned)
        self._counts = {}
        self._armed = False
        self._launched = 0
        self._pads_epoch = -1
        self._sq = torch.zeros(len(self.buckets), 2, device=flat.device)
        self.comm_stream = torch.cuda.Stream(device=flat.device)
        self.lo, self.hi = 0, 0  # the owned elements are self.slices, not one range
        for p in flat.params:
            p.__dict__["_tt_grad_ready"] = self._on_grad_ready

    def begin_micro_step(self, last: bool) -> None:
        """Trainer hook before each micro-step's forward.  The last micro-step of a step
        launches each bucket's reduce-scatter as soon as its gradients are final; the
        others count the gradient notifications so the last one knows when that is."""
        if self.buckets is None:
            return
        if last and self._counts:
            self._expected = dict(self._counts)
        self._armed = last and self._expected is not None
        self._counts = {}
        self._launched = 0
        self._ready = [False] * len(self.buckets)

    def _on_grad_ready(self, p) -> None:
        k = id(p)
        self._counts[k] = self._counts.get(k, 0) + 1
        if not self._armed:
            return
        b = self._bucket_of[k]
        if all(self._counts.get(id(q), 0) >= self._expected.get(id(q), 1) for q in self._bucket_params[b]):
            self._ready[b] = True
            while self._launched < len(self.buckets) and self._ready[self._launched]:
                self._launch_bucket(self._launched, overlap=True)
                self._launched += 1

    def _launch_bucket(self, b: int, overlap: bool) -> None:
        lo, hi = self.slices[b]
        heap = self.flat.heap
        if not overlap:
            heap.reduce_scatter_bucket(self.flat.grad, lo, hi, self.flat.dense_numel, 1.0 / self.dp, self._sq[b],
                                       max_blocks=1 << 30)
            return
        main = torch.cuda.current_stream(self.flat.device)
        self.comm_stream.wait_stream(main)  # this bucket's gradients are written (stream order)
        with torch.cuda.stream(self.comm_stream):
            heap.reduce_scatter_bucket(self.flat.grad, lo, hi, self.flat.dense_numel, 1.0 / self.dp, self._sq[b],
                                       max_blocks=32)

    def _finish_buckets(self) -> None:
        main = torch.cuda.current_stream(self.flat.device)
        if self._armed:
            while self._launched < len(self.buckets):  # anything the notifications did not cover
                self._launch_bucket(self._launched, overlap=True)
                self._launched += 1
            main.wait_stream(self.comm_stream)
        else:
            for b in range(len(self.buckets)):
                self._launch_bucket(b, overlap=False)
        self._armed = False
        self._pads_epoch = self.flat.heap.publish_sumsq(self._sq)

    # ---------------------------------------------------------------- gradient sync
    @torch.no_grad()
    def reduce_gradients(self):
        g = self.flat.grad
        if self.buckets is not None:
            self._finish_buckets()
            return
        if self.sp > 1 and self.flat.dense_numel > 0:
            dist.all_reduce(g[:self.flat.dense_numel], op=dist.ReduceOp.SUM, group=self.sp_group)
        if self.native:
            # dense_numel is a multiple of the flat layout's 64-element alignment
            self.flat.heap.reduce_scatter_sumsq(g, self.lo, self.hi, self.flat.dense_numel, 1.0 / self.dp)
            return
        if self.dp > 1:
            if dist.get_backend(self.dp_group) == "nccl":
                dist.reduce_scatter_tensor(g[self.lo:self.hi], g, op=dist.ReduceOp.AVG, group=self.dp_group)
            else:  # gloo: no AVG and no aliasing of output into input
                out = torch.empty(self.shard, dtype=g.dtype, device=g.device)
                dist.reduce_scatter_tensor(out, g, op=dist.ReduceOp.SUM, group=self.dp_group)
                g[self.lo:self.hi].copy_(out.div_(self.dp))

    # ---------------------------------------------------------------- norm
    @torch.no_grad()
    def grad_norm_and_coef(self, max_norm: float):
        if self.native:
            # The norm and clip coefficient are formed inside the update kernel from the
            # sums of squares every rank published; they land in _normc after step().
            self._max_norm = float(max_norm)
            return self._normc[0], None
        g = self.flat.grad[self.lo:self.hi]
        dense_hi = max(self.lo, min(self.hi, self.flat.dense_numel))
        if g.is_cuda:
            from tinytron_b200.ops import _ext

            C = _ext.load()
            C.sumsq(self.flat.grad[self.lo:dense_hi], self._sq[0:1], self._scratch, False)
            C.sumsq(self.flat.grad[dense_hi:self.hi], self._sq[1:2], self._scratch, False)
        else:
            self._sq[0] = self.flat.grad[self.lo:dense_hi].double().pow(2).sum().float()
            self._sq[1] = self.flat.grad[dense_hi:self.hi].double().pow(2).sum().float()
        if self.dp > 1:
            dist.all_reduce(self._sq, op=dist.ReduceOp.SUM, group=self.dp_group)
        if self.sp > 1 and self.flat.dense_numel < self.flat.numel:
            dist.all_reduce(self._sq[1:2], op=dist.ReduceOp.SUM, group=self.sp_group)
        total_sq = self._sq.sum().reshape(1)
        if g.is_cuda:
            _ext.load().clip_coef(total_sq, self._norm, self._coef, float(max_norm))
        else:
            self._norm.copy_(total_sq.sqrt())
            self._coef.copy_(torch.clamp(max_norm / (self._norm + 1e-6), max=1.0))
        return self._norm[0], self._coef

    # ---------------------------------------------------------------- update
    @torch.no_grad()
    def step(self, lr: float | None = None, grad_scale: torch.Tensor | None = None):
        grp = self.param_groups[0]
        lr = grp["lr"] if lr is None else lr
        b1, b2 = grp["betas"]
        self.step_count += 1
        lo, hi = self.lo, self.hi
        if self.buckets is not None:
            heap = self.flat.heap
            for (slo, shi), (m0, m1) in zip(self.slices, self.state_off):
                heap.adamw_allgather(self.flat.data, self.flat.grad, self.flat.bf16, self.exp_avg[m0:m1],
                                     self.exp_avg_sq[m0:m1], slo, shi, lr, (b1, b2), grp["eps"], grp["weight_decay"],
                                     self.step_count, self._max_norm, norm_out=self._normc,
                                     pads_epoch=self._pads_epoch)
            if self.flat.bf16 is not None:  # waits for every peer's stores, then all shadows
                heap.shadow_refresh(self.flat.data, self.flat.bf16, 0, 0)
            self.flat.mark_shadows_fresh()
            return
        if self.native:
            heap = self.flat.heap
            heap.adamw_allgather(self.flat.data, self.flat.grad, self.flat.bf16, self.exp_avg, self.exp_avg_sq, lo, hi,
                                 lr, (b1, b2), grp["eps"], grp["weight_decay"], self.step_count, self._max_norm,
                                 norm_out=self._normc)
            if self.flat.bf16 is not None:
                heap.shadow_refresh(self.flat.data, self.flat.bf16, lo, hi)
            self.flat.mark_shadows_fresh()
            return
        p = self.flat.data[lo:hi]
        g = self.flat.grad[lo:hi]
        if p.is_cuda:
            from tinytron_b200.ops import _ext

            _ext.load().adamw_step(p, g, self.exp_avg, self.exp_avg_sq,
                                   self.flat.bf16[lo:hi] if self.flat.bf16 is not None else None, lr, b1, b2,
                                   grp["eps"], grp["weight_decay"], self.step_count, grad_scale)
        else:
            gg = g * grad_scale if grad_scale is not None else g
            p.mul_(1 - lr * grp["weight_decay"])
            self.exp_avg.lerp_(gg, 1 - b1)
            self.exp_avg_sq.mul_(b2).addcmul_(gg, gg, value=1 - b2)
            bc1 = 1 - b1 ** self.step_count
            bc2 = 1 - b2 ** self.step_count
            denom = (self.exp_avg_sq.sqrt() / math.sqrt(bc2)).add_(grp["eps"])
            p.addcdiv_(self.exp_avg, denom, value=-lr / bc1)
            if self.flat.bf16 is not None:
                self.flat.bf16[lo:hi].copy_(p)
        if self.dp > 1:
            if dist.get_backend(self.dp_group) == "nccl":
                dist.all_gather_into_tensor(self.flat.data, self.flat.data[lo:hi], group=self.dp_group)
            else:
                dist.all_gather_into_tensor(self.flat.data, self.flat.data[lo:hi].clone(), group=self.dp_group)
            if self.flat.bf16 is not None:
                # shadow of the shards other ranks updated
                if lo > 0:
                    self.flat.bf16[:lo].copy_(self.flat.data[:lo])
                if hi < self.flat.numel:
                    self.flat.bf16[hi:].copy_(self.flat.data[hi:])
        self.flat.mark_shadows_fresh()

    def zero_grad(self, set_to_none: bool = True):
        self.flat.zero_grad()

    # ---------------------------------------------------------------- state
    def _owned(self) -> list:
        return [list(x) for x in self.slices] if self.buckets is not None else [[self.lo, self.hi]]

    def state_dict(self):
        return {"step": self.step_count, "exp_avg": self.exp_avg, "exp_avg_sq": self.exp_avg_sq,
                "param_groups": [dict(g) for g in self.param_groups], "shard": self._owned(),
                "numel": self.flat.numel, "format": "tinytron_b200.flat_zero1.v2"}

    def load_state_dict(self, sd):
        if sd.get("numel") != self.flat.numel or [list(x) for x in sd.get("shard", [])] != self._owned():
            raise ValueError("optimizer state layout does not match the current flat layout")
        self.step_count = int(sd["step"])
        self.exp_avg.copy_(sd["exp_avg"])
        self.exp_avg_sq.copy_(sd["exp_avg_sq"])
        for g, s in zip(self.param_groups, sd["param_groups"]):
            g.update(s)
