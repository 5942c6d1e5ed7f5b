"""Parallelism: process groups, DDP/ZeRO-1 gradient and parameter sync, Ulysses SP,
expert-parallel all-to-all (reference API: tinytron/distributed/__init__.py:1-6)."""
from . import parallel_state
from .expert_parallel import ep_all_to_all, ep_all_to_all_no_grad
from .ulysses import allreduce_non_expert_grads_across_sp, ulysses_all_to_all


def __getattr__(name):
    if name in ("DistributedOptimizer", "partition_tensors"):
        from . import zero1

        return getattr(zero1, name)
    raise AttributeError(name)


__all__ = ["parallel_state", "DistributedOptimizer", "partition_tensors", "ulysses_all_to_all",
           "allreduce_non_expert_grads_across_sp", "ep_all_to_all", "ep_all_to_all_no_grad"]
