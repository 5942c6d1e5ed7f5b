"""Symmetric device heap over NVLink (Python side of ``csrc/runtime/comm.cu``).

A :class:`SymmetricHeap` is one device buffer per rank of a process group, mapped
into every other rank through CUDA IPC, so kernels can load from and store to
peers' memory directly.  Tensors are carved from the heap by a bump allocator;
ranks that make the same ``alloc`` calls in the same order get the same offsets,
which is what makes the heap *symmetric* (a peer's copy of a tensor lives at the
same offset of the peer's heap).

The collectives on the heap replace the reference's NCCL calls on the hot paths:

* :meth:`SymmetricHeap.all_reduce` — one-shot all-reduce of a heap tensor (inference
  row-parallel outputs; reference ``model/modules/attn.py:364``, ``mlp.py:221``).
* :meth:`SymmetricHeap.reduce_scatter_sumsq` and :meth:`SymmetricHeap.adamw_allgather`
  — the ZeRO-1 gradient reduce-scatter (with the clip norm's sums of squares) and
  the fused clip + AdamW + parameter all-gather (reference: DDP all-reduce in
  ``training/trainer.py:214-220`` plus the per-tensor broadcasts of
  ``distributed/zero1/distributed_optimizer.py:106-119``).

Every device-side wait is bounded (``TT_COMM_TIMEOUT_S``, default 60 s); a wait
that gives up records a status code and the host raises from
:func:`tinytron_b200.ops.check_status`.

Single-GPU test mode (:meth:`SymmetricHeap.create_emulated`): W heaps on one
device act as the W ranks of one group; the collectives are launched rank by rank
with waits disabled, so no kernel ever waits for another.
"""
from __future__ import annotations

import socket

import torch
import torch.distributed as dist

ALIGN = 256


def _C():
    from tinytron_b200.ops import _ext

    return _ext.load()


def _dtype_code(dtype: torch.dtype) -> int:
    # c10::ScalarType enum values (stable public ABI of torch)
    return {torch.uint8: 0, torch.int32: 3, torch.int64: 4, torch.float16: 5, torch.float32: 6,
            torch.bfloat16: 15}[dtype]


def same_host(group) -> bool:
    """True when every rank of ``group`` runs on this host (CUDA IPC needs that)."""
    names = [None] * dist.get_world_size(group)
    dist.all_gather_object(names, socket.gethostname(), group=group)
    return len(set(names)) == 1


class SymmetricHeap:
    def __init__(self, gid: int, nbytes: int, rank: int, world: int, device: torch.device):
        self.gid = gid
        self.nbytes = nbytes
        self.rank = rank
        self.world = world
        self.device = device
        self._next = int(_C().comm_user_offset())
        self._base = int(_C().comm_heap_base(gid))
        self._closed = False

    # ------------------------------------------------------------------ construction
    @classmethod
    def create(cls, nbytes: int, group=None, device=None) -> "SymmetricHeap":
        """Collective over ``group``: allocate this rank's heap and map every peer's."""
        C = _C()
        device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        world = dist.get_world_size(group)
        rank = dist.get_rank(group)
        if world > 8:
            raise ValueError("SymmetricHeap supports at most 8 ranks (one NVLink domain)")
        nbytes = int(nbytes) + int(C.comm_user_offset())
        gid = int(C.comm_create(device.index, nbytes))
        h = C.comm_ipc_handle(gid)
        handles = [None] * world
        dist.all_gather_object(handles, bytes(h.tolist()), group=group)
        table = torch.tensor([list(x) for x in handles], dtype=torch.uint8)
        C.comm_open(gid, rank, world, table)
        heap = cls(gid, nbytes, rank, world, device)
        dist.barrier(group=group)
        return heap

    @classmethod
    def create_emulated(cls, nbytes: int, world: int, device=None, waits: bool = False) -> list["SymmetricHeap"]:
        """W heaps on one device acting as the W ranks of one group (tests)."""
        C = _C()
        device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        nbytes = int(nbytes) + int(C.comm_user_offset())
        gids = [int(C.comm_create(device.index, nbytes)) for _ in range(world)]
        C.comm_open_emulated(gids, waits)
        return [cls(g, nbytes, r, world, device) for r, g in enumerate(gids)]

    # ------------------------------------------------------------------ memory
    def alloc(self, shape, dtype: torch.dtype, zero: bool = True) -> torch.Tensor:
        shape = tuple(int(s) for s in (shape if isinstance(shape, (tuple, list)) else (shape,)))
        numel = 1
        for s in shape:
            numel *= s
        nb = numel * torch.empty((), dtype=dtype).element_size()
        off = self._next
        if off + nb > self.nbytes:
            raise MemoryError(f"symmetric heap exhausted ({off + nb} > {self.nbytes} bytes)")
        self._next = (off + nb + ALIGN - 1) // ALIGN * ALIGN
        t = _C().comm_view(self.gid, off, list(shape), _dtype_code(dtype))
        if zero:
            t.zero_()
        return t

    def offset_of(self, t: torch.Tensor) -> int:
        off = t.data_ptr() - self._base
        if not (0 <= off and off + t.numel() * t.element_size() <= self.nbytes):
            raise ValueError("tensor does not live in this symmetric heap")
        return off

    @staticmethod
    def bytes_needed(*specs) -> int:
        """Heap bytes for a list of (numel, dtype) allocations."""
        total = 0
        for numel, dtype in specs:
            nb = int(numel) * torch.empty((), dtype=dtype).element_size()
            total += (nb + ALIGN - 1) // ALIGN * ALIGN
        return total

    # ------------------------------------------------------------------ collectives
    def barrier(self) -> None:
        from tinytron_b200.utils.watchdog import fault_active

        # TT_FAULT_INJECT=skip_signal@R: rank R waits without signalling, so its peers'
        # bounded device waits expire with a status code (host-side injection).
        signal = not fault_active("skip_signal", dist.get_rank() if dist.is_initialized() else self.rank)
        _C().comm_barrier(self.gid, signal)

    def all_reduce(self, src: torch.Tensor, out: torch.Tensor | None = None,
                   residual: torch.Tensor | None = None) -> torch.Tensor:
        """out = sum over ranks of ``src`` (a heap tensor) (+ residual); one-shot, every
        rank gets the bit-identical sum (same rank order everywhere).  The caller must
        not overwrite ``src`` before the *next* collective on this heap has started on
        every rank; alternating two source buffers satisfies that."""
        out = torch.empty_like(src) if out is None else out
        _C().comm_all_reduce(self.gid, self.offset_of(src), out, residual)
        return out

    def reduce_scatter_sumsq(self, grad: torch.Tensor, lo: int, hi: int, split: int, scale: float) -> None:
        """grad[lo:hi] = scale * sum over ranks of grad[lo:hi] (in place); publishes this
        rank's sums of squares of the reduced shard (split at ``split``) to every peer."""
        _C().comm_reduce_scatter_sumsq(self.gid, self.offset_of(grad), int(lo), int(hi), int(split), float(scale))

    def adamw_allgather(self, data: torch.Tensor, grad: torch.Tensor, p16: torch.Tensor | None, m: torch.Tensor,
                        v: torch.Tensor, lo: int, hi: int, lr: float, betas, eps: float, wd: float, step: int,
                        max_norm: float, norm_out: torch.Tensor | None = None,
                        extra_sq: torch.Tensor | None = None, pads_epoch: int = -1) -> None:
        _C().comm_adamw_allgather(self.gid, self.offset_of(data), self.offset_of(grad), p16, m, v, int(lo), int(hi),
                                  float(lr), float(betas[0]), float(betas[1]), float(eps), float(wd), int(step),
                                  float(max_norm), extra_sq, norm_out, int(pads_epoch))

    def reduce_scatter_bucket(self, grad: torch.Tensor, lo: int, hi: int, split: int, scale: float,
                              sq_local: torch.Tensor, max_blocks: int = 32) -> None:
        """One bucket of an overlapped reduce-scatter: grad[lo:hi] = scale * sum over ranks
        (in place); the slice's sums of squares go to ``sq_local`` (fp32 [2]) on this rank."""
        _C().comm_reduce_scatter_bucket(self.gid, self.offset_of(grad), int(lo), int(hi), int(split), float(scale),
                                        sq_local, int(max_blocks))

    def publish_sumsq(self, sq: torch.Tensor) -> int:
        """Publish the total of per-bucket sums of squares ([n, 2]) to every peer; returns
        the epoch the update kernels must wait for."""
        return int(_C().comm_publish_sumsq(self.gid, sq))

    def all_to_all(self, slot: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
        """out[c] = chunk ``rank`` of rank c's ``slot`` (both [world, ...], equal chunks)."""
        _C().comm_all_to_all(self.gid, self.offset_of(slot), out)
        return out

    def shadow_refresh(self, data: torch.Tensor, p16: torch.Tensor, lo: int, hi: int) -> None:
        _C().comm_shadow_refresh(self.gid, self.offset_of(data), p16, int(lo), int(hi))

    def replay_slots(self, slot_bytes: int) -> tuple[torch.Tensor, int]:
        """Two adjacent slots of ``slot_bytes`` (a multiple of 256) for the replayable
        collectives; returns (buffer, slot_bytes)."""
        slot_bytes = (int(slot_bytes) + ALIGN - 1) // ALIGN * ALIGN
        return self.alloc(2 * slot_bytes, torch.uint8), slot_bytes

    def replay_publish(self, slots: torch.Tensor, slot_bytes: int, x: torch.Tensor) -> None:
        """Step 1 of a graph-safe collective: copy ``x`` into this rank's current slot and
        signal the peers (the epoch lives on the device, so a CUDA graph may hold this)."""
        _C().comm_replay_publish(self.gid, self.offset_of(slots), int(slot_bytes), x)

    def replay_reduce(self, slots: torch.Tensor, slot_bytes: int, out: torch.Tensor,
                      residual: torch.Tensor | None = None, root: int = -1) -> torch.Tensor:
        """Step 2: wait for every peer's publish, then out = sum over ranks (or the ``root``
        rank's input) (+ residual); bit-identical on every rank (fixed rank order)."""
        _C().comm_replay_reduce(self.gid, self.offset_of(slots), int(slot_bytes), out, residual, int(root))
        return out

    @property
    def epoch(self) -> int:
        return int(_C().comm_epoch(self.gid))

    def close(self) -> None:
        """Free the heap (collective in spirit: peers must be done with it).  Tensors
        carved from it must not be used afterwards."""
        if not self._closed:
            _C().comm_destroy(self.gid)
            self._closed = True


# ---------------------------------------------------------------------------- row-parallel all-reduce
class RowParallelAllReduce:
    """Inference row-parallel all-reduce over a SEP group on a symmetric heap (replaces
    the reference's ``dist.all_reduce`` of c_proj / MoE partial outputs,
    ``model/modules/attn.py:364``, ``mlp.py:221``).  Graph-safe: both of its kernels take
    their epoch from device memory, so the decode step that contains it can be captured
    in one CUDA graph and replayed (the two heap slots alternate with the epoch's parity,
    which is what makes one wait per call enough)."""

    def __init__(self, group, max_numel: int, device=None):
        self.max_numel = int(max_numel)
        nbytes = self.max_numel * 2
        self.heap = SymmetricHeap.create(2 * ((nbytes + ALIGN - 1) // ALIGN * ALIGN), group, device)
        self.slots, self.slot_bytes = self.heap.replay_slots(nbytes)

    def fits(self, numel: int) -> bool:
        return numel <= self.max_numel and numel % 8 == 0

    def publish_target(self) -> tuple[int, int, int]:
        """(heap id, slot offset, slot bytes) for a producer kernel that writes its result
        into this rank's slot and signals the peers itself (the fused publish); only
        :meth:`reduce_into` has to follow."""
        return self.heap.gid, self.heap.offset_of(self.slots), self.slot_bytes

    def reduce_into(self, out: torch.Tensor) -> None:
        self.heap.replay_reduce(self.slots, self.slot_bytes, out.view(-1))

    def __call__(self, y: torch.Tensor) -> torch.Tensor | None:
        n = y.numel()
        if y.dtype != torch.bfloat16 or n > self.max_numel or not y.is_cuda or n % 8:
            return None
        y = y.contiguous()
        out = torch.empty_like(y)
        self.heap.replay_publish(self.slots, self.slot_bytes, y.view(-1))
        self.heap.replay_reduce(self.slots, self.slot_bytes, out.view(-1))
        return out

    def close(self):
        self.heap.close()


_ROW_AR: dict = {}


def enable_row_parallel_all_reduce(group, max_numel: int, device=None) -> RowParallelAllReduce:
    """Collective over ``group``: route :func:`row_parallel_all_reduce` on this group
    through a symmetric heap of ``max_numel`` bf16 elements per slot."""
    key = id(group)
    ar = _ROW_AR.get(key)
    if ar is None or ar.max_numel < max_numel:
        if ar is not None:
            ar.close()
        ar = RowParallelAllReduce(group, max_numel, device)
        _ROW_AR[key] = ar
    return ar


def disable_row_parallel_all_reduce(group) -> None:
    ar = _ROW_AR.pop(id(group), None)
    if ar is not None:
        ar.close()


def row_parallel_heap_enabled(group) -> bool:
    return id(group) in _ROW_AR


def row_parallel_target(group) -> RowParallelAllReduce | None:
    """The group's heap all-reduce, for producers that publish into it themselves."""
    return _ROW_AR.get(id(group))


def row_parallel_all_reduce(y: torch.Tensor, group) -> torch.Tensor:
    """SUM over ``group``: the symmetric-heap kernel when enabled for the group (and y
    fits), else NCCL in place."""
    ar = _ROW_AR.get(id(group))
    if ar is not None:
        out = ar(y)
        if out is not None:
            return out
    dist.all_reduce(y, op=dist.ReduceOp.SUM, group=group)
    return y


# ---------------------------------------------------------------------------- all-to-all
class HeapAllToAll:
    """Equal-split all-to-all over a group on a symmetric heap (Ulysses head<->sequence
    exchange; reference ``distributed/sequence_parallel/ulysses.py:7-22``).  The caller
    writes its outgoing chunks into :meth:`slot` (e.g. ``torch.stack(..., out=slot)``)
    and calls :meth:`exchange`.  Two slots alternate, so one start barrier per call
    suffices (a slot is rewritten only after every peer started the next exchange)."""

    def __init__(self, group, device=None):
        self.group = group
        self.device = device
        self.heap = None
        self.cap = 0
        self.slots = None
        self.i = 0

    def _ensure(self, nbytes: int):
        if self.heap is None or nbytes > self.cap:  # collective: same sizes on every rank
            if self.heap is not None:
                self.heap.close()
            cap = max(nbytes, 1 << 20)
            self.heap = SymmetricHeap.create(2 * ((cap + ALIGN - 1) // ALIGN * ALIGN), self.group, self.device)
            self.slots = [self.heap.alloc(cap, torch.uint8, zero=False), self.heap.alloc(cap, torch.uint8, zero=False)]
            self.cap = cap

    def slot(self, shape, dtype) -> torch.Tensor:
        numel = 1
        for s in shape:
            numel *= int(s)
        nbytes = numel * torch.empty((), dtype=dtype).element_size()
        self._ensure(nbytes)
        return self.slots[self.i][:nbytes].view(dtype).view(tuple(shape))

    def exchange(self, slot: torch.Tensor) -> torch.Tensor:
        out = torch.empty_like(slot)
        self.heap.all_to_all(slot, out)
        self.i ^= 1
        return out


class UlyssesExchange:
    """Send slots and the device-epoch protocol of the fused Ulysses kernels
    (``csrc/runtime/ulysses.cu``) for one SEP group.  The heap grows (collectively: every
    rank asks for the same sizes in the same order) when a larger exchange is needed."""

    def __init__(self, group, device=None):
        self.group = group
        self.device = device
        self.heap = None
        self.slots = None
        self.slot_bytes = 0

    def ensure(self, nbytes: int):
        if self.heap is None or nbytes > self.slot_bytes:
            if self.heap is not None:
                torch.cuda.synchronize()
                self.heap.close()
            cap = max(int(nbytes), 1 << 20)
            cap = (cap + ALIGN - 1) // ALIGN * ALIGN
            self.heap = SymmetricHeap.create(2 * cap + ALIGN, self.group, self.device)
            self.slots, self.slot_bytes = self.heap.replay_slots(cap)
        return self.heap.gid, self.heap.offset_of(self.slots), self.slot_bytes

    def close(self):
        if self.heap is not None:
            self.heap.close()
            self.heap = None


_UL: dict = {}


def ulysses_exchange_for(group) -> UlyssesExchange | None:
    return _UL.get(id(group))


_A2A: dict = {}


def enable_heap_all_to_all(group, device=None) -> HeapAllToAll:
    """Route the SEP group's all-to-alls through symmetric heaps: the generic equal-split
    exchange and the fused Ulysses head<->sequence kernels."""
    a = _A2A.get(id(group))
    if a is None:
        a = HeapAllToAll(group, device)
        _A2A[id(group)] = a
    if id(group) not in _UL:
        _UL[id(group)] = UlyssesExchange(group, device)
    return a


def heap_all_to_all_for(group) -> HeapAllToAll | None:
    return _A2A.get(id(group))
