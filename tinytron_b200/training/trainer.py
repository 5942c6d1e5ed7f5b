"""Trainer (reference: tinytron/training/trainer.py:48-571).

Same construction order, overridable hooks (``_init_dataset``, ``_init_optimizer``,
``_next_train_batch``, ``_resume_from_checkpoint``, ``save``), loss weighting,
cosine LR schedule, log line format and checkpoint files as the reference.

The step itself is B200-native: fp32 master weights live in flat buffers with a
bf16 shadow for the tensor cores; weight gradients accumulate in fp32 inside the
GEMM epilogues across micro-steps; the gradient sync is one SP all-reduce of the
non-expert prefix plus one DP reduce-scatter (ZeRO-1); clipping is a fused norm
and the update is one fused AdamW kernel over the owned shard followed by an
all-gather.  There is no host synchronisation inside a step.
"""
from __future__ import annotations

import math
import os
import random
import time
from contextlib import contextmanager, nullcontext
from datetime import timedelta
from itertools import islice

import numpy as np
import torch
import torch.distributed as dist
from torch.utils.data import DataLoader
from torch.utils.data.distributed import DistributedSampler

from tinytron_b200.models import GPT
from tinytron_b200.parallel import parallel_state
from tinytron_b200.parallel.buffers import FlatParams
from tinytron_b200.parallel.zero1 import FlatZeRO1
from tinytron_b200.utils import compute_mfu, get_model_params, get_training_info, set_seed
from tinytron_b200.utils.profile import nvtx_range

from .config import Config
from .data import MockDataset, build_lm_collate_fn


def _group_size(g) -> int:
    return dist.get_world_size(g) if g is not None else 1


class Trainer:
    def __init__(self, config: Config):
        self.config = config
        self._init_distributed(config)
        tb, b, t = config.train.total_batch_size, config.train.batch_size, config.train.seq_len
        assert tb % (b * t * self.dp_world_size) == 0, (
            f"make sure total_batch_size {tb} is divisible by batch_size {b} * seq_len {t} * "
            f"dp_world_size {self.dp_world_size}")
        if self.master_process and config.logging.print_config:
            print(f"Training config: {config.as_dict()}")
        self._init_dataset(config)
        self.training_info = get_training_info(self.num_train_samples, t, tb, b, self.dp_world_size,
                                               config.train.max_steps, config.train.max_epochs)
        if config.optim.warmup_steps >= self.training_info["max_steps"]:
            raise ValueError(f"warmup_steps must be < max_steps. Got warmup_steps={config.optim.warmup_steps}, "
                             f"max_steps={self.training_info['max_steps']}.")
        if self.master_process:
            print(f"The training process will train {self.training_info['epochs']} epochs, "
                  f"{self.training_info['max_steps']} steps.")
            print(f"=> total tokens per step: {tb}")
            print(f"=> calculated gradient accumulation steps: {self.training_info['grad_accum_steps']}")
        self._init_model(config)
        self._init_optimizer(config)
        self._init_logging(config)
        self.one_step_results = {}

    # ------------------------------------------------------------------ setup
    def _init_distributed(self, config: Config):
        self.rank = int(os.environ.get("RANK", 0))
        self.local_rank = int(os.environ.get("LOCAL_RANK", 0))
        self.world_size = int(os.environ.get("WORLD_SIZE", 1))
        self.device = torch.device("cuda", self.local_rank) if torch.cuda.is_available() else torch.device("cpu")
        if self.device.type == "cuda":
            torch.cuda.set_device(self.device)
        self._owns_pg = False
        if not dist.is_initialized() and (self.world_size > 1 or "MASTER_ADDR" in os.environ):
            backend = config.parallel.backend if self.device.type == "cuda" else "gloo"
            timeout = timedelta(seconds=int(os.environ.get("TT_PG_TIMEOUT_S", "600")))
            kw = {"device_id": self.device} if backend == "nccl" else {}
            dist.init_process_group(backend=backend, init_method=config.parallel.init_method, timeout=timeout, **kw)
            self._owns_pg = True
        set_seed(config.seed.seed + self.rank, deterministic=config.seed.deterministic)
        self.master_process = self.rank == 0
        parallel_state.set_comm_impl(config.parallel.comm_impl)
        if dist.is_initialized():
            parallel_state.initialize_model_parallel(config.parallel)
            parallel_state.print_model_parallel_topology(self.master_process and config.logging.print_config,
                                                         tag="Init Distributed Topology")
        self.dp_group = parallel_state.get_dp_group_or_none()
        self.sp_group = parallel_state.get_sp_group_or_none()
        self.dp_sp_group = parallel_state._DP_SP_GROUP
        self.dp_rank = parallel_state.get_dp_rank()
        self.dp_world_size = parallel_state.get_dp_world_size()
        self.sp_rank = parallel_state.get_sp_rank()
        self.sp_world_size = parallel_state.get_sp_world_size()
        self.dp_sp_rank = parallel_state.get_dp_sp_rank()
        self.dp_sp_world_size = parallel_state.get_dp_sp_world_size()

    def _init_dataset(self, config: Config):
        if not config.data.use_mock_data:
            raise NotImplementedError("Only --use_mock_data is built in; override _init_dataset for real data "
                                      "(the reference ships the same placeholder).")
        self.train_dataset = MockDataset(config.data.mock_data_num_samples, config.train.seq_len,
                                         vocab_size=config.model.vocab_size, deterministic=config.seed.deterministic,
                                         base_seed=config.seed.seed)
        self.val_dataset = (MockDataset(config.data.mock_data_num_samples // 10, config.train.seq_len,
                                        vocab_size=config.model.vocab_size, deterministic=config.seed.deterministic,
                                        base_seed=config.seed.seed, seed_offset=1_000_000_000)
                            if config.train.do_val else None)
        self.train_sampler = DistributedSampler(self.train_dataset, num_replicas=self.dp_world_size,
                                                rank=self.dp_rank, shuffle=True)
        collate = self._build_lm_collate_fn(config)
        pin = config.data.pin_memory and self.device.type == "cuda"
        self.train_loader = DataLoader(self.train_dataset, batch_size=config.train.batch_size,
                                       sampler=self.train_sampler, num_workers=config.data.num_workers,
                                       pin_memory=pin, collate_fn=collate)
        if self.val_dataset is not None:
            self.val_sampler = DistributedSampler(self.val_dataset, num_replicas=self.dp_world_size,
                                                  rank=self.dp_rank, shuffle=False)
            self.val_loader = DataLoader(self.val_dataset, batch_size=config.train.batch_size,
                                         sampler=self.val_sampler, num_workers=config.data.num_workers,
                                         pin_memory=pin, collate_fn=collate)
        else:
            self.val_loader = None
        self.num_train_samples = len(self.train_dataset)
        self.train_sampler_epoch = 0
        self.train_loader_iter_idx = 0
        self.train_sampler.set_epoch(0)
        self.train_loader_iter = enumerate(self.train_loader)

    def _build_lm_collate_fn(self, config: Config):
        return build_lm_collate_fn(config.train.seq_len, self.sp_world_size)

    def _init_model(self, config: Config):
        self.model_config = config.model
        model = GPT(self.model_config, device=self.device)
        if self.master_process and config.logging.print_config:
            print(f"Params config: {get_model_params(self.model_config)}")
        self.model = model
        self.raw_model = model
        pad = max(1, self.dp_world_size) * 64
        heap_factory = None
        if self._use_native_comm(config):
            from tinytron_b200.parallel.symm import SymmetricHeap

            def heap_factory(nbytes):
                return SymmetricHeap.create(nbytes, group=self.dp_group, device=self.device)
        self.flat = FlatParams(model, pad_to_multiple=pad, with_bf16=self.device.type == "cuda",
                               heap_factory=heap_factory)
        if (self.device.type == "cuda" and self.sp_world_size > 1 and parallel_state.native_comm_enabled()
                and self.sp_world_size <= 8):
            from tinytron_b200.parallel.symm import enable_heap_all_to_all, same_host

            if same_host(self.sp_group):  # Ulysses exchanges by NVLink peer loads
                enable_heap_all_to_all(self.sp_group, self.device)

    def _use_native_comm(self, config: Config) -> bool:
        """ZeRO-1 gradient/parameter sync over NVLink peer memory (tt_comm) instead of
        NCCL: CUDA, DP > 1 inside one node, AdamW with the distributed optimizer.
        ``--comm_impl nccl`` (or ``TT_NATIVE_COMM=0``) selects the NCCL path."""
        if self.device.type != "cuda" or self.dp_world_size <= 1 or not parallel_state.native_comm_enabled():
            return False
        if not (config.parallel.use_distributed_optimizer and config.optim.optimizer == "adam"):
            return False
        if self.dp_world_size > 8:
            return False
        from tinytron_b200.parallel.symm import same_host

        return same_host(self.dp_group)

    def _init_optimizer(self, config: Config):
        o = config.optim
        self.use_flat_optimizer = o.optimizer == "adam"
        if self.use_flat_optimizer:
            shard = config.parallel.use_distributed_optimizer
            self.optimizer = FlatZeRO1(self.flat, dp_group=self.dp_group if shard else None, sp_group=self.sp_group,
                                       lr=o.max_lr, betas=(o.adam_beta1, o.adam_beta2), eps=o.adam_eps,
                                       weight_decay=o.weight_decay,
                                       bucket_bytes=max(0, config.parallel.grad_bucket_mb) << 20)
            self.raw_optimizer = self.optimizer
            self._replicated_dp = (not shard) and self.dp_world_size > 1
            return
        from tinytron_b200.optim import Muon

        muon_params, adam_params = [], []
        for name, p in self.raw_model.named_parameters():
            if not p.requires_grad:
                continue
            if p.ndim == 2 and "wte" not in name and "lm_head" not in name:
                muon_params.append(p)
            else:
                adam_params.append(p)
        groups = [
            {"params": muon_params, "use_muon": True, "use_adam": False, "lr": o.max_lr,
             "momentum": o.muon_momentum, "weight_decay": o.weight_decay},
            {"params": adam_params, "use_muon": False, "use_adam": True, "lr": o.max_lr,
             "betas": (o.adam_beta1, o.adam_beta2), "eps": o.adam_eps, "weight_decay": o.weight_decay},
        ]
        opt = Muon(groups)
        if config.parallel.use_distributed_optimizer and self.dp_sp_world_size > 1:
            # ZeRO-1 over each tensor's replica group: dense matrices over DP x SEP, expert
            # matrices over DP; one Newton-Schulz per matrix in the whole job
            from tinytron_b200.optim.muon import DistributedMuon

            self.optimizer = DistributedMuon(opt, self.flat, dense_group=self.dp_sp_group, expert_group=self.dp_group)
            self.raw_optimizer = self.optimizer.optimizer
        else:
            self.optimizer = opt
            self.raw_optimizer = opt

    def _init_profiler(self, config: Config):
        @contextmanager
        def dummy(name):
            yield

        if config.train.use_profiler:
            s0, s1 = config.train.steps_to_profile[0], config.train.steps_to_profile[1]
            assert s0 >= 1, "steps_to_profile[0] should be >= 1"

            def handler(prof):
                if self.master_process:
                    prof.export_chrome_trace(f"{self.log_dir}/rank{self.rank}_trace.json")

            acts = [torch.profiler.ProfilerActivity.CPU]
            if self.device.type == "cuda":
                acts.append(torch.profiler.ProfilerActivity.CUDA)
            self.profiler = torch.profiler.profile(
                schedule=torch.profiler.schedule(wait=s0 - 1, warmup=1, active=s1 + 1 - s0, repeat=1),
                on_trace_ready=handler, record_shapes=True, with_stack=True, with_flops=True, activities=acts)
        else:
            self.profiler = None
        self.profiler_record_fn = torch.profiler.record_function if config.train.use_profiler else dummy

    def _init_logging(self, config: Config):
        n = sum(p.numel() for p in self.flat.params)
        self.log_dir = os.path.join(config.logging.log_dir,
                                    f"modelsize_{n}_lr{config.optim.max_lr}_BS{config.train.batch_size}_"
                                    f"SL{config.train.seq_len}_DP{self.dp_world_size}_SEP{self.sp_world_size}_")
        self.log_file = os.path.join(self.log_dir, "log.txt")
        if self.master_process:
            os.makedirs(self.log_dir, exist_ok=True)
            open(self.log_file, "w").close()
        if dist.is_initialized():
            dist.barrier()
        self.profiler = None
        self.profiler_record_fn = lambda name: nullcontext()

    # ------------------------------------------------------------------ schedule
    def _lr_scheduler(self, it: int, max_steps: int, warmup_steps: int, max_lr: float, min_lr: float) -> float:
        if it < warmup_steps:
            return max_lr * (it + 1) / warmup_steps
        if it > max_steps:
            return min_lr
        ratio = (it - warmup_steps) / (max_steps - warmup_steps)
        assert 0 <= ratio <= 1
        return min_lr + 0.5 * (1.0 + math.cos(math.pi * ratio)) * (max_lr - min_lr)

    def _autocast_context(self, precision: str):
        # The CUDA kernels already run bf16 operands with fp32 accumulation and fp32
        # masters (the semantics of the reference's bf16 autocast); fp32 on CPU.
        if precision == "fp16":
            raise NotImplementedError("FP16 precision is not supported yet")
        return nullcontext()

    # ------------------------------------------------------------------ step
    def _prepare_local_batch(self, data_batch: dict):
        x, y = data_batch["input_ids"], data_batch["labels"]
        T = x.shape[1]
        assert T % self.sp_world_size == 0, "sequence length must be divisible by sp_world_size"
        c = T // self.sp_world_size
        x = x[:, self.sp_rank * c:(self.sp_rank + 1) * c]
        y = y[:, self.sp_rank * c:(self.sp_rank + 1) * c]
        nb = self.device.type == "cuda"
        return x.to(self.device, non_blocking=nb), y.to(self.device, non_blocking=nb)

    def _one_training_micro_step(self, config: Config, micro_step: int, data_batch: dict):
        x, y = self._prepare_local_batch(data_batch)
        valid = (y != -100).sum()
        with self.profiler_record_fn("forward"):
            with self._autocast_context(config.train.precision):
                _, loss, logging_loss = self.model(x.reshape(x.shape[0], -1), y.reshape(y.shape[0], -1))
        # SP-group and global valid-token counts, reduced inside the model's forward together
        # with its other statistics (one packed collective per micro-step)
        tok, tok_all = self.raw_model.last_token_counts
        weight = (tok * self.dp_world_size / tok_all.clamp(min=1.0)).reshape(())
        ga = self.training_info["grad_accum_steps"]
        loss = loss * weight.to(loss.dtype) / ga
        with self.profiler_record_fn("backward"):
            loss.backward()
        return logging_loss.detach() * weight / ga, valid

    def _collect_cpu_grads(self):
        """CPU path: autograd wrote p.grad; fold into the flat fp32 grad buffer."""
        for p in self.flat.params:
            if p.grad is not None:
                p.__dict__["main_grad"].add_(p.grad)
                p.grad = None

    def _sync_and_clip(self, max_norm: float):
        if self.device.type != "cuda":
            self._collect_cpu_grads()
        if self.use_flat_optimizer:
            opt = self.optimizer
            if getattr(self, "_replicated_dp", False):
                if self.sp_world_size > 1:
                    dist.all_reduce(self.flat.grad[:self.flat.dense_numel], group=self.sp_group)
                self.flat.grad.div_(self.dp_world_size)
                dist.all_reduce(self.flat.grad, group=self.dp_group)
            else:
                opt.reduce_gradients()
            norm, coef = opt.grad_norm_and_coef(max_norm)
            return norm, coef
        # Muon path: SP sum of the dense grads, DP average, then the global norm from two
        # flat sums of squares (expert part summed over EP); the clip coefficient is
        # applied by the optimizer to the gradients it uses (on their owners).
        g = self.flat.grad
        if self.sp_world_size > 1:
            dist.all_reduce(g[:self.flat.dense_numel], op=dist.ReduceOp.SUM, group=self.sp_group)
        if self.dp_world_size > 1:
            g.div_(self.dp_world_size)
            dist.all_reduce(g, op=dist.ReduceOp.SUM, group=self.dp_group)
        self.flat.expose_grads()
        return self._flat_clip_coef(max_norm)

    def _flat_clip_coef(self, max_norm: float):
        """(global grad norm, clip coefficient) as device scalars, after the gradient sync."""
        g, split = self.flat.grad, self.flat.dense_numel
        sq = torch.zeros(2, device=g.device, dtype=torch.float32)
        if g.is_cuda:
            from tinytron_b200.ops import _ext

            C = _ext.load()
            scratch = torch.empty(4096, device=g.device)
            C.sumsq(g[:split], sq[0:1], scratch, False)
            C.sumsq(g[split:], sq[1:2], scratch, False)
        else:
            sq[0] = g[:split].double().pow(2).sum().float()
            sq[1] = g[split:].double().pow(2).sum().float()
        if self.sp_world_size > 1 and split < self.flat.numel:
            dist.all_reduce(sq[1:2], op=dist.ReduceOp.SUM, group=self.sp_group)
        norm = sq.sum().sqrt()
        coef = torch.clamp(max_norm / (norm + 1e-6), max=1.0)
        return norm, coef

    def _one_training_step(self, config: Config, step: int):
        self.model.train()
        self.flat.zero_grad()
        loss_accum = torch.zeros((), device=self.device)
        valid_accum = torch.zeros((), device=self.device, dtype=torch.long)
        ga = self.training_info["grad_accum_steps"]
        begin = getattr(self.optimizer, "begin_micro_step", None)
        for micro in range(ga):
            if begin is not None:  # overlapped reduce-scatter: armed for the last micro-step
                begin(micro == ga - 1)
            batch = self._next_train_batch()
            ll, v = self._one_training_micro_step(config, micro, batch)
            loss_accum += ll
            valid_accum += v
        with nvtx_range("grad_sync_clip"):
            norm, coef = self._sync_and_clip(config.train.grad_clip_value)
        lr = self._lr_scheduler(step, self.training_info["max_steps"], config.optim.warmup_steps,
                                config.optim.max_lr, config.optim.min_lr)
        if self.use_flat_optimizer:
            self.optimizer.step(lr=lr, grad_scale=coef)
        else:
            for g in self.optimizer.param_groups:
                g["lr"] = lr
            self.optimizer.step(grad_scale=coef)
            for p in self.flat.params:
                p.grad = None
            self.flat.refresh_bf16() if self.device.type == "cuda" else None
        if self.dp_sp_world_size > 1:
            # one packed collective for the step's loss (identical across SP ranks, so its
            # DP x SP sum / (DP x SP) is the DP mean) and the global valid-token count
            from tinytron_b200.parallel.scalars import all_reduce_scalars

            red = all_reduce_scalars(torch.stack([loss_accum.float(), valid_accum.float()]), self.dp_sp_group)
            loss_accum = red[0] / self.dp_sp_world_size
            valid_accum = red[1].round().long()
        self.one_step_results["lr"] = lr
        self.one_step_results["loss"] = loss_accum
        self.one_step_results["grad_norm"] = norm
        self.one_step_results["valid_tokens"] = valid_accum

    def train_step(self, step: int) -> dict:
        """Public single-step API: runs one optimizer step (all micro-steps) and returns
        the step results (device tensors; no host sync)."""
        self.one_step_results = {}
        self._one_training_step(self.config, step)
        return self.one_step_results

    def _next_train_batch(self):
        try:
            idx, batch = next(self.train_loader_iter)
        except StopIteration:
            self.train_sampler_epoch += 1
            self.train_loader_iter_idx = 0
            self.train_sampler.set_epoch(self.train_sampler_epoch)
            self.train_loader_iter = enumerate(self.train_loader)
            idx, batch = next(self.train_loader_iter)
        self.train_loader_iter_idx = idx + 1
        return batch

    # ------------------------------------------------------------------ loop
    def _init_heartbeat(self):
        """Heartbeat watchdog (``TT_HEARTBEAT_TIMEOUT_S`` > 0 and more than one rank):
        a silent or failed peer is reported between steps as PeerFailure."""
        timeout = float(os.environ.get("TT_HEARTBEAT_TIMEOUT_S", "0") or 0)
        if timeout <= 0 or not dist.is_initialized() or dist.get_world_size() <= 1:
            return None
        from tinytron_b200.utils.watchdog import Heartbeat

        return Heartbeat(dist.get_rank(), dist.get_world_size(), interval=min(1.0, timeout / 4), timeout=timeout)

    def train(self):
        self.heartbeat = self._init_heartbeat()
        try:
            self._train_loop()
        except BaseException:
            if self.heartbeat is not None:
                self.heartbeat.close(exit_code=1)
                self.heartbeat = None
            raise
        if self.heartbeat is not None:
            self.heartbeat.close(exit_code=0)
            self.heartbeat = None

    def _train_loop(self):
        from tinytron_b200.utils.watchdog import fault_point

        self.results = {}
        self._resume_from_checkpoint()
        self._init_profiler(self.config)
        if self.profiler:
            self.profiler.start()
        cfg = self.config
        max_steps = self.training_info["max_steps"]
        for step in range(self.start_step, max_steps):
            fault_point("exit", self.rank, step)  # host-side fault injection (tests)
            if self.heartbeat is not None:
                self.heartbeat.check()  # before this step launches any kernel or collective
            self.one_step_results = {}
            t0 = time.time()
            last = step == max_steps - 1
            dev_timing = self.device.type == "cuda" and os.environ.get("TT_DEVICE_TIMING", "0") == "1"
            if dev_timing:
                ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                ev0.record()
            with self.profiler_record_fn("training_step"), nvtx_range(f"step{step}"):
                self._one_training_step(cfg, step)
            if dev_timing:
                ev1.record()
            if self.device.type == "cuda":
                torch.cuda.synchronize()
            if dev_timing:  # device time of the step, max over ranks (same collective on every rank)
                dev_ms = torch.tensor([ev0.elapsed_time(ev1)], device=self.device)
                if dist.is_initialized() and dist.get_world_size() > 1:
                    dist.all_reduce(dev_ms, op=dist.ReduceOp.MAX)
                self.one_step_results["device_ms"] = float(dev_ms.item())
            if self.profiler:
                self.profiler.step()
            if not cfg.train.debug and cfg.train.do_val and (step % cfg.train.val_every_steps == 0 or last):
                self.eval()
                if self.master_process:
                    v = self.one_step_results["val_loss"].item()
                    print(f"validation loss: {v:.4f}")
                    with open(self.log_file, "a") as f:
                        f.write(f"{step} val {v:.4f}\n")
            if cfg.ckpt.do_save and not cfg.train.debug and step > 0 and (step % cfg.ckpt.save_every_steps == 0 or last):
                self.save(step)
            dt = time.time() - t0
            tokens = int(self.one_step_results.get("valid_tokens", torch.tensor(0)).item())
            if tokens <= 0:
                tokens = cfg.train.batch_size * cfg.train.seq_len * self.training_info["grad_accum_steps"] * \
                    self.dp_world_size
            tps = tokens / dt
            mfu, _, _ = compute_mfu(self.raw_model, cfg.train.batch_size, cfg.train.seq_len, dt,
                                    self.training_info["grad_accum_steps"], dtype="bf16") \
                if self.device.type == "cuda" else (0.0, 0.0, 0.0)
            if self.master_process and (step % cfg.logging.log_every == 0 or last):
                loss = self.one_step_results["loss"].item()
                gn = float(self.one_step_results["grad_norm"])
                print(f"step {step:5d}/{max_steps} | loss: {loss:.6f} | lr {self.one_step_results['lr']:.4e} | "
                      f"grad norm: {gn:.4f} | dt: {dt * 1000:.2f}ms | tok/sec: {tps:.2f} | MFU: {mfu * 100:.2f}%"
                      + (f" | device: {self.one_step_results['device_ms']:.2f}ms"
                         if "device_ms" in self.one_step_results else ""), flush=True)
                with open(self.log_file, "a") as f:
                    f.write(f"{step} train {loss:.6f}\n")
            self.results[step] = self.one_step_results
        if self.profiler:
            self.profiler.stop()
        self.close()

    def close(self):
        hb = getattr(self, "heartbeat", None)
        if hb is not None:  # clean exit published before the store may go away
            hb.close(exit_code=0)
            self.heartbeat = None
        if self._owns_pg and dist.is_initialized():
            dist.barrier()
            dist.destroy_process_group()
            parallel_state.destroy_model_parallel()
            self._owns_pg = False

    @torch.no_grad()
    def eval(self):
        self.model.eval()
        loss_sum = torch.zeros((), device=self.device)
        tokens = torch.zeros((), device=self.device)
        for batch in self.val_loader:
            x, y = self._prepare_local_batch(batch)
            _, _, ll = self.model(x, y)
            t = (y != -100).sum().float()
            if self.sp_world_size > 1:
                dist.all_reduce(t, group=self.sp_group)
            loss_sum += ll * t
            tokens += t
        if self.dp_world_size > 1:
            dist.all_reduce(loss_sum, group=self.dp_group)
            dist.all_reduce(tokens, group=self.dp_group)
        self.one_step_results["val_loss"] = loss_sum / tokens.clamp(min=1.0)
        self.model.train()

    # ------------------------------------------------------------------ checkpoint
    def save(self, step: int | None = None):
        from . import checkpoint as ck

        prefix = os.path.join(self.log_dir, f"{step:05d}")
        os.makedirs(f"{prefix}_rng", exist_ok=True)
        ck.save_optimizer_state(self.raw_optimizer, prefix, self.rank)
        rng = {"torch": torch.get_rng_state(), "numpy": np.random.get_state(), "python": random.getstate()}
        if self.device.type == "cuda":
            rng["cuda"] = torch.cuda.get_rng_state(self.local_rank)
        torch.save(rng, os.path.join(f"{prefix}_rng", f"rank{self.rank}.pt"))
        ck.save_local_model_shard(self.raw_model, prefix, self.rank)
        if dist.is_initialized():
            dist.barrier()
        if self.master_process:
            ck.save_rank0_legacy_model(self.raw_model, prefix)
            meta = {
                "config": self.config.as_dict(),
                "step": step,
                "this_step_results": {k: (v.detach().cpu() if torch.is_tensor(v) else v)
                                      for k, v in self.one_step_results.items()},
                "opt_part_assignment": getattr(self.optimizer, "part_assignment", None),
                "model_layout": ck.model_layout_metadata(),
                "model_sharded": True,
                "model_shard_pattern": f"{step:05d}_model_rank{{rank:05d}}.pt",
                "sampler_state": {"epoch": self.train_sampler_epoch, "iter_idx": self.train_loader_iter_idx},
                "rng_state": rng,
            }
            meta.update(self._checkpoint_extra_meta())
            torch.save(meta, ck.checkpoint_meta_path(prefix))
            ck.write_checksums(prefix)
        if dist.is_initialized():
            dist.barrier()

    def _checkpoint_extra_meta(self) -> dict:
        """Extra entries for the checkpoint's ``_meta.pt`` (subclass hook, e.g. a data position)."""
        return {}

    def _resume_from_checkpoint(self):
        from . import checkpoint as ck

        ckpt_dir = self.config.ckpt.resume_path or self.log_dir
        prefix = ck.find_latest_checkpoint_prefix(ckpt_dir)
        if prefix is None:
            self.start_step = 0
            return
        meta = torch.load(ck.checkpoint_meta_path(prefix), map_location="cpu", weights_only=False)
        self._resumed_meta = meta
        sd = ck.load_model_state_dict_for_training(prefix, self.model_config, self.rank, meta)
        self.raw_model.load_state_dict(sd)
        if self.device.type == "cuda":
            self.flat.refresh_bf16()
        if ck.training_layout_matches_current(meta):
            ck.load_optimizer_state(self.raw_optimizer, prefix, self.rank)
        elif self.master_process:
            print("=> Skipping optimizer restore because checkpoint model_layout differs from current layout.")
        ss = meta.get("sampler_state", {})
        epoch, it = int(ss.get("epoch", 0)), int(ss.get("iter_idx", 0))
        self.train_sampler_epoch, self.train_loader_iter_idx = epoch, it
        if self.train_sampler is not None:
            self.train_sampler.set_epoch(epoch)
            self.train_loader_iter = enumerate(islice(self.train_loader, it, None), start=it)
        step = meta.get("step")
        self.start_step = (step + 1) if step is not None else 0
        if self.master_process:
            print(f"=> Resumed from {ckpt_dir} | next_step={self.start_step}, sampler_epoch={epoch}, "
                  f"dataloader_iter_idx={it}")
        rng_path = f"{prefix}_rng/rank{self.rank}.pt"
        if os.path.exists(rng_path):
            rng = torch.load(rng_path, map_location="cpu", weights_only=False)
            torch.set_rng_state(rng["torch"].to(torch.uint8).cpu())
            if "cuda" in rng and self.device.type == "cuda":
                torch.cuda.set_rng_state(rng["cuda"].to(torch.uint8).cpu(), self.local_rank)
            np.random.set_state(rng["numpy"])
            if "python" in rng:
                random.setstate(rng["python"])
        if dist.is_initialized():
            dist.barrier()
