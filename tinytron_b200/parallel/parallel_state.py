"""Process-group layout for DP x SEP (reference: tinytron/distributed/parallel_state.py:14-336).

Layout (identical to the reference so checkpoints and samplers line up):
  * SEP group i  = ranks [i*S, ..., i*S + S - 1]  (contiguous; one data replica)
  * DP group j   = ranks [j, S + j, 2S + j, ...]   (same offset across SEP groups)
  * DP_SP group  = the whole world
SP and EP are aliases of SEP.  ``dp_rank == global_rank // S``.

Unlike the reference, every getter also works without an initialised process
group (world size 1, rank 0, group None), so single-device and CPU paths need no
``init_process_group``.  ``get_*_group`` still asserts when groups are expected
but missing, as in the reference.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

_SEP_GROUP = None
_DP_GROUP = None
_DP_SP_GROUP = None
_SEP_SIZE = None
_DP_SIZE = None
_DP_SP_SIZE = None
# Collective implementation for the training/inference hot paths: "native" runs them as
# peer loads/stores on symmetric heaps (one node), "nccl" keeps every collective on NCCL.
_COMM_IMPL = "native"
_SEP_RANKS: list[int] | None = None
_DP_RANKS: list[int] | None = None


def initialize_model_parallel(config=None, sep_size: int | None = None, timeout=None) -> None:
    """Build SEP / DP / world groups.  Call after ``dist.init_process_group``.

    ``config`` is a ``ParallelConfig`` (anything with ``sep_size``); ``sep_size``
    may be given directly instead.
    """
    global _SEP_GROUP, _DP_GROUP, _DP_SP_GROUP, _SEP_SIZE, _DP_SIZE, _DP_SP_SIZE, _SEP_RANKS, _DP_RANKS
    if sep_size is None:
        sep_size = int(getattr(config, "sep_size", 1))
    assert dist.is_initialized(), "Must initialize PyTorch distributed environment first!"
    world = dist.get_world_size()
    rank = dist.get_rank()
    assert world % sep_size == 0, "World size must be divisible by sep_size"
    dp_size = world // sep_size
    _SEP_SIZE, _DP_SIZE, _DP_SP_SIZE = sep_size, dp_size, world
    kw = {} if timeout is None else {"timeout": timeout}
    for i in range(dp_size):
        ranks = list(range(i * sep_size, (i + 1) * sep_size))
        g = dist.new_group(ranks, **kw)
        if rank in ranks:
            _SEP_GROUP, _SEP_RANKS = g, ranks
    for j in range(sep_size):
        ranks = [i * sep_size + j for i in range(dp_size)]
        g = dist.new_group(ranks, **kw)
        if rank in ranks:
            _DP_GROUP, _DP_RANKS = g, ranks
    _DP_SP_GROUP = dist.new_group(list(range(world)), **kw)


def destroy_model_parallel() -> None:
    global _SEP_GROUP, _DP_GROUP, _DP_SP_GROUP, _SEP_SIZE, _DP_SIZE, _DP_SP_SIZE, _SEP_RANKS, _DP_RANKS
    from .scalars import release_scalar_reducers

    release_scalar_reducers()
    _SEP_GROUP = _DP_GROUP = _DP_SP_GROUP = None
    _SEP_SIZE = _DP_SIZE = _DP_SP_SIZE = None
    _SEP_RANKS = _DP_RANKS = None


def model_parallel_is_initialized() -> bool:
    return _SEP_GROUP is not None


def _world_rank() -> int:
    return dist.get_rank() if dist.is_available() and dist.is_initialized() else 0


# ------------------------------------------------------------------ DP
def get_dp_group():
    assert _DP_GROUP is not None, "DP Group is not initialized"
    return _DP_GROUP


def get_dp_world_size() -> int:
    return _DP_SIZE if _DP_SIZE is not None else 1


def get_dp_rank() -> int:
    if _DP_GROUP is None:
        return 0
    return dist.get_rank(group=_DP_GROUP)


def get_dp_global_rank(group_rank: int | None = None) -> int:
    if group_rank is None:
        group_rank = get_dp_rank()
    if _DP_GROUP is None:
        return group_rank
    return dist.get_global_rank(_DP_GROUP, group_rank)


def _get_dp_group_id_from_layout(global_rank: int, sep_size: int) -> int:
    return global_rank % sep_size


# ------------------------------------------------------------------ SEP (= SP = EP)
def get_sep_group():
    assert _SEP_GROUP is not None, "SEP Group is not initialized"
    return _SEP_GROUP


def get_sep_world_size() -> int:
    return _SEP_SIZE if _SEP_SIZE is not None else 1


def get_sep_rank() -> int:
    if _SEP_GROUP is None:
        return 0
    return dist.get_rank(group=_SEP_GROUP)


def get_sep_global_rank(group_rank: int | None = None) -> int:
    if group_rank is None:
        group_rank = get_sep_rank()
    if _SEP_GROUP is None:
        return group_rank
    return dist.get_global_rank(_SEP_GROUP, group_rank)


def get_sep_ranks() -> list[int]:
    return list(_SEP_RANKS) if _SEP_RANKS is not None else [_world_rank()]


def get_dp_ranks() -> list[int]:
    return list(_DP_RANKS) if _DP_RANKS is not None else [_world_rank()]


def _get_sep_group_id_from_layout(global_rank: int, sep_size: int) -> int:
    return global_rank // sep_size


get_sp_group = get_sep_group
get_sp_world_size = get_sep_world_size
get_sp_rank = get_sep_rank
get_sp_global_rank = get_sep_global_rank
get_ep_group = get_sep_group
get_ep_world_size = get_sep_world_size
get_ep_rank = get_sep_rank
get_ep_global_rank = get_sep_global_rank


def get_sp_group_or_none():
    return _SEP_GROUP


def get_dp_group_or_none():
    return _DP_GROUP


# ------------------------------------------------------------------ world
def get_dp_sp_group():
    assert _DP_SP_GROUP is not None, "DP_SP Group is not initialized"
    return _DP_SP_GROUP


def get_dp_sp_world_size() -> int:
    return _DP_SP_SIZE if _DP_SP_SIZE is not None else 1


def get_dp_sp_rank() -> int:
    if _DP_SP_GROUP is None:
        return 0
    return dist.get_rank(group=_DP_SP_GROUP)


def get_dp_sp_global_rank(group_rank: int | None = None) -> int:
    if group_rank is None:
        group_rank = get_dp_sp_rank()
    if _DP_SP_GROUP is None:
        return group_rank
    return dist.get_global_rank(_DP_SP_GROUP, group_rank)


def print_model_parallel_topology(master_process: bool, tag: str = "Parallel Topology", group_for_gather=None,
                                  only_rank0: bool = True, flush: bool = True) -> None:
    """Print the static rank table and each rank's own view of its groups
    (gathered to rank 0), like reference parallel_state.py:143-336."""
    assert dist.is_initialized(), "torch.distributed must be initialized before printing topology"
    assert _SEP_GROUP is not None and _DP_GROUP is not None, "call initialize_model_parallel() first"
    world, rank = dist.get_world_size(), dist.get_rank()
    S, D = get_sep_world_size(), get_dp_world_size()
    group_for_gather = group_for_gather or get_dp_sp_group()
    payload = [rank, _get_sep_group_id_from_layout(rank, S), get_sep_rank(), S,
               _get_dp_group_id_from_layout(rank, S), get_dp_rank(), D]
    payload += [get_sep_global_rank(i) for i in range(S)] + [get_dp_global_rank(i) for i in range(D)]
    dev = torch.device("cuda", torch.cuda.current_device()) if (
        torch.cuda.is_available() and dist.get_backend(group_for_gather) == "nccl") else torch.device("cpu")
    t = torch.tensor(payload, dtype=torch.int64, device=dev)
    gathered = [torch.empty_like(t) for _ in range(world)]
    dist.all_gather(gathered, t, group=group_for_gather)
    if (only_rank0 and rank != 0) or not master_process:
        return
    p = lambda *a: print(*a, flush=flush)  # noqa: E731
    p(f"\n=== {tag} ===")
    p(f"world_size={world}, sep_size={S}, dp_size={D} | layout: SEP=rows(contiguous), DP=cols(same offset)")
    p("\n[Static Rank Mapping]")
    p(f"{'global':>6} | {'sep_gid(data_rep)':>16} | {'sep_rank':>8} | {'dp_gid':>6} | {'dp_rank':>7}")
    for r in range(world):
        p(f"{r:>6} | {r // S:>16} | {r % S:>8} | {r % S:>6} | {r // S:>7}")
    p("\n[Grid View] rows=SEP groups (data replicas), cols=SEP ranks")
    for i in range(D):
        p(f"SEP[{i:>2}] | " + " ".join(f"{i * S + j:>5}" for j in range(S)))
    p("\n[Dynamic Per-Rank View (gathered)]")
    for row in sorted((g.cpu().tolist() for g in gathered), key=lambda v: v[0]):
        p(f"rank {row[0]:>3}: sep_gid={row[1]} sep={row[2]}/{row[3]} dp_gid={row[4]} dp={row[5]}/{row[6]} "
          f"sep_members={row[7:7 + S]} dp_members={row[7 + S:7 + S + D]}")
    p("=" * (len(tag) + 8))


def set_comm_impl(impl: str) -> None:
    """Select the collective implementation (``--comm_impl``): "native" or "nccl"."""
    global _COMM_IMPL
    if impl not in ("native", "nccl"):
        raise ValueError(f"Unsupported comm_impl: {impl}")
    _COMM_IMPL = impl


def native_comm_enabled() -> bool:
    """True when the symmetric-heap collectives are selected.  ``TT_NATIVE_COMM=0`` in the
    environment forces NCCL for callers that do not go through the trainer's flags."""
    import os

    return _COMM_IMPL == "native" and os.environ.get("TT_NATIVE_COMM", "1") != "0"
