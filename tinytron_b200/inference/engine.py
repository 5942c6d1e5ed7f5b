"""KV-cache inference engine (reference: tinytron/inference/engine.py:16-261).

Same constructor and ``generate`` signature/return values as the reference.
Differences that matter for speed:
  * prefill computes logits only for the last position (the reference materialises
    [B, T, V] logits and slices the last row);
  * the EOS stop test is evaluated on the device and read back every
    ``eos_check_interval`` steps; the returned sequences are cut at the exact step
    where every sequence had produced EOS, so the output equals the per-step check;
  * with SEP > 1 every rank samples by itself and no token is broadcast: the row-parallel
    all-reduces sum in the same rank order on every rank, so all ranks hold bit-identical
    logits, and the sampler's seeds come from a CPU generator whose seed SEP rank 0 sends
    once per ``generate`` call, so every rank draws the same tokens (the reference lets
    SEP rank 0 sample and broadcasts every step's tokens);
  * on CUDA with the paged (or contiguous) cache, pages for the whole generation are
    mapped up front and one decode step (embedding -> every layer's fused RoPE/append
    + split-KV attention -> LM head) is captured in a CUDA graph and replayed, so a
    decode step costs one graph launch instead of hundreds of kernel launches from
    Python; with SEP > 1 the row-parallel all-reduces run on a symmetric heap.
"""
from __future__ import annotations

import time

import torch
import torch.distributed as dist

from tinytron_b200.models import GPT
from tinytron_b200.parallel import parallel_state

from .cache import PagedKVCache
from .checkpoint import load_model_state_dict_for_inference
from .sampler import sample_next_token, sample_next_token_with_log_prob


class InferenceEngine:
    def __init__(self, model_config, checkpoint_path: str | None = None, device: str = "cuda",
                 dtype: torch.dtype = torch.bfloat16, use_paged_kv_cache: bool = True, kv_cache_page_size: int = 128,
                 eos_check_interval: int = 8, use_cuda_graph: bool = True):
        self.device = torch.device(device)
        if self.device.type == "cuda":
            if self.device.index is None:
                self.device = torch.device("cuda", torch.cuda.current_device())
            torch.cuda.set_device(self.device)
        self.model_config = model_config
        self.use_paged_kv_cache = use_paged_kv_cache
        self.kv_cache_page_size = kv_cache_page_size
        self.eos_check_interval = max(1, int(eos_check_interval))
        self.model = GPT(model_config, device=self.device)
        if checkpoint_path:
            self.model.load_state_dict(load_model_state_dict_for_inference(checkpoint_path, model_config))
        self.model.eval()
        self.dtype = dtype
        self.use_cuda_graph = use_cuda_graph and self.device.type == "cuda"
        self._graph = None

    def _graph_ok(self) -> bool:
        """A decode step is capturable when nothing in it synchronises with the host.  With
        SEP > 1 that needs the row-parallel all-reduces on the symmetric heap (their epochs
        live on the device); the MoE local-expert path is device-only."""
        if not self.use_cuda_graph:
            return False
        sep = self._sep()
        if sep is None:
            return True
        from tinytron_b200.parallel.symm import row_parallel_heap_enabled

        return row_parallel_heap_enabled(sep[0])

    def _enable_heap_all_reduce(self, B: int, T: int) -> None:
        sep = self._sep()
        if sep is None or self.device.type != "cuda":
            return
        from tinytron_b200.parallel.symm import enable_row_parallel_all_reduce, same_host

        if same_host(sep[0]):
            enable_row_parallel_all_reduce(sep[0], B * T * self.model_config.hidden_size, self.device)

    def _capture_decode(self, cache, B: int):
        """Capture one decode step at the cache's current length; returns
        (graph, static token input [B, 1], static logits [B, 1, V])."""
        L = cache.current_length
        static_tok = torch.zeros(B, 1, dtype=torch.long, device=self.device)
        # one eager warm-up step outside the graph (allocations, lazy tables), then rewind
        self.model._forward_cached(static_tok, cache, True, L, last_only=True)
        cache.set_length(L)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            static_logits, _ = self.model._forward_cached(static_tok, cache, True, L, last_only=True)
        cache.set_length(L)  # capture advanced the host length without running anything
        torch.cuda.synchronize()
        return g, static_tok, static_logits

    def _decode_graph_loop(self, logits, cache, tokens, B: int, P: int, n_new: int, temperature, top_k, top_p,
                           want_lp: bool, gen):
        """Every decode step as ONE graph replay: the forward of the last token, the draw and
        the token write all run on the device (the draw's seed and Philox offset live in a
        device tensor that the step advances), so the host only launches the graph.  The
        first token is drawn eagerly from the prefill logits with the same kernels.
        Returns (steps, log-probs [B, steps] or None, the graph; the caller releases it after
        synchronising)."""
        from tinytron_b200.ops import _ext

        from .sampler import _cuda_sample

        C = _ext.load()
        dev = self.device
        base = int(torch.randint(0, 2 ** 62, (1,), generator=gen).item())  # same on every SEP rank
        rng = torch.tensor([base, 0], dtype=torch.long, device=dev)
        tok_in = torch.zeros(B, 1, dtype=torch.long, device=dev)
        nxt = torch.empty(B, dtype=torch.long, device=dev)
        lp = torch.empty(B, dtype=torch.float32, device=dev) if want_lp else None
        lp_all = torch.empty(B, n_new, dtype=torch.float32, device=dev) if want_lp else None

        def draw(lg):
            _cuda_sample(lg[:, -1, :], temperature, top_k, top_p, want_lp, rng=rng, out=(nxt, lp))
            C.decode_advance(nxt, tokens, P, tok_in.view(-1), rng, lp, lp_all)

        draw(logits)  # token 0
        L = cache.current_length
        # one eager forward outside the graph (allocations, lazy tables), then rewind
        self.model._forward_cached(tok_in, cache, True, L, last_only=True)
        cache.set_length(L)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            lg, _ = self.model._forward_cached(tok_in, cache, True, L, last_only=True)
            draw(lg)
        cache.set_length(L)  # capture advanced the host length without running anything
        for _ in range(n_new - 1):
            g.replay()
        for c in cache._layer_caches:  # the replays advanced the device lengths
            c.current_length += n_new - 1
            c.seq_lens = [c.current_length] * c.batch_size
        return n_new, lp_all, g

    # ------------------------------------------------------------------ SEP-synced sampling
    def _sep(self):
        g = parallel_state.get_sp_group_or_none()
        if g is None or not dist.is_initialized() or parallel_state.get_sep_world_size() <= 1:
            return None
        return g, parallel_state.get_sep_rank(), parallel_state.get_sep_global_rank(0)

    def _sampling_generator(self):
        """CPU generator for the sampler's seeds.  Without SEP: None (torch's global RNG, as
        before).  With SEP: one seed drawn by SEP rank 0 and sent once per generate call, so
        every rank's draws are identical (one small collective per call, none per step)."""
        sep = self._sep()
        if sep is None:
            return None
        g, r, src = sep
        seed = torch.randint(0, 2 ** 62, (1,), dtype=torch.long)
        dev = self.device if dist.get_backend(g) == "nccl" else torch.device("cpu")
        seed = seed.to(dev)
        dist.broadcast(seed, src=src, group=g)
        return torch.Generator().manual_seed(int(seed.item()))

    def _sample_next_token_synced(self, logits, temperature=1.0, top_k=None, top_p=None, generator=None):
        return sample_next_token(logits, temperature=temperature, top_k=top_k, top_p=top_p, generator=generator)

    def _sample_next_token_with_log_prob_synced(self, logits, temperature=1.0, top_k=None, top_p=None,
                                                generator=None):
        return sample_next_token_with_log_prob(logits, temperature=temperature, top_k=top_k, top_p=top_p,
                                               generator=generator)

    def new_cache(self, batch_size: int, max_seq_len: int | None = None):
        if self.use_paged_kv_cache:
            return PagedKVCache.from_model_config(self.model_config, batch_size, self.kv_cache_page_size, self.device,
                                                  self.dtype, max_seq_len=max_seq_len)
        return PagedKVCache.contiguous(self.model_config, batch_size, self.device, self.dtype, max_seq_len=max_seq_len)

    # ------------------------------------------------------------------ generation
    @torch.no_grad()
    def generate(self, input_ids: torch.Tensor, max_new_tokens: int, temperature: float = 1.0, top_k=None,
                 top_p=None, eos_token_id: int | None = None, return_stats: bool = False,
                 return_logprobs: bool = False):
        if input_ids.dim() != 2:
            raise ValueError(f"input_ids must be [B, T], got shape={tuple(input_ids.shape)}")
        prompt = input_ids.to(self.device)
        B, P = prompt.shape
        total = P + max_new_tokens
        if total > self.model_config.block_size:
            raise ValueError(f"Requested total sequence length {total} exceeds block_size {self.model_config.block_size}")
        tokens = torch.empty(B, total, dtype=prompt.dtype, device=self.device)
        tokens[:, :P] = prompt
        cache = self.new_cache(B, max_seq_len=total)
        cuda = self.device.type == "cuda"
        if cuda:
            cache.reserve(total)
            self._enable_heap_all_reduce(B, P)
        graph = None
        gen = self._sampling_generator()
        sync = torch.cuda.synchronize if cuda else (lambda *a: None)
        logp_steps = []
        finished = torch.zeros(B, dtype=torch.bool, device=self.device)
        all_done = []
        sync()
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)] if cuda else None
        if ev:
            ev[0].record()
        t0 = time.perf_counter()
        logits, cache = self.model._forward_cached(prompt, cache, True, 0, last_only=True)
        if ev:
            ev[1].record()
        sync()
        t1 = time.perf_counter()
        cur = P
        steps = 0
        stop_at = None
        lp_graph = None
        graph_loop = (cuda and eos_token_id is None and max_new_tokens > 2 and self._graph_ok()
                      and tokens.dtype == torch.long)
        if graph_loop:
            steps, lp_graph, graph = self._decode_graph_loop(logits, cache, tokens, B, P, max_new_tokens, temperature,
                                                             top_k, top_p, return_logprobs, gen)
            cur = P + steps
        for i in range(0 if graph_loop else max_new_tokens):
            last = logits[:, -1, :]
            if return_logprobs:
                nxt, lp = self._sample_next_token_with_log_prob_synced(last, temperature, top_k, top_p, gen)
                logp_steps.append(lp)
            else:
                nxt = self._sample_next_token_synced(last, temperature, top_k, top_p, gen)
            tokens[:, cur] = nxt
            cur += 1
            steps += 1
            if eos_token_id is not None:
                finished |= nxt == eos_token_id
                all_done.append(finished.all())
                if steps % self.eos_check_interval == 0 or i == max_new_tokens - 1:
                    flags = torch.stack(all_done[-self.eos_check_interval:]).tolist()
                    if any(flags):
                        stop_at = steps - len(flags) + flags.index(True) + 1
                        break
            if i == max_new_tokens - 1:
                break
            if graph is None and cuda and self._graph_ok() and max_new_tokens - i > 2:
                graph = self._capture_decode(cache, B)
            if graph is not None:
                g, static_tok, static_logits = graph
                static_tok.copy_(nxt.unsqueeze(-1))
                g.replay()
                for c in cache._layer_caches:  # the graph advanced the device lengths
                    c.current_length += 1
                    c.seq_lens = [c.current_length] * c.batch_size
                logits = static_logits
            else:
                logits, cache = self.model._forward_cached(nxt.unsqueeze(-1), cache, True, cur - 1, last_only=True)
        if ev:
            ev[2].record()
        sync()
        t2 = time.perf_counter()
        if stop_at is not None:
            steps = stop_at
            cur = P + stop_at
            logp_steps = logp_steps[:stop_at]
        tokens = tokens[:, :cur]
        if not return_stats and not return_logprobs:
            return tokens
        extras = {}
        if return_stats:
            dt_p, dt_d = max(t1 - t0, 1e-9), max(t2 - t1, 1e-9)
            extras.update({"prefill_tokens_per_sec": B * P / dt_p,
                           "decode_tokens_per_sec": (B * steps / dt_d) if steps else 0.0,
                           "prefill_tokens": float(B * P), "decode_tokens": float(B * steps)})
            if ev:  # the same phases timed on the device (CUDA events on the generating stream)
                dp_ms, dd_ms = ev[0].elapsed_time(ev[1]), ev[1].elapsed_time(ev[2])
                extras.update({"prefill_ms_device": dp_ms, "decode_ms_device": dd_ms,
                               "prefill_tokens_per_sec_device": B * P / max(dp_ms, 1e-6) * 1e3,
                               "decode_tokens_per_sec_device": (B * steps / max(dd_ms, 1e-6) * 1e3) if steps else 0.0})
        if return_logprobs:
            if lp_graph is not None:
                lp = lp_graph
            else:
                lp = torch.stack(logp_steps, 1) if logp_steps else torch.empty(B, 0, device=self.device)
            extras.update({"prompt_len": float(P), "decode_steps": float(steps), "token_log_probs": lp,
                           "response_mask": torch.ones_like(lp, dtype=torch.float32)})
        return tokens, extras
