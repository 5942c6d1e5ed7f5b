"""Sampling (reference: tinytron/inference/sampler.py:6-61): temperature, top-k,
top-p (nucleus, always keeping the most likely token), multinomial draw, and the
log-prob of the drawn token under the filtered distribution."""
from __future__ import annotations

import torch


def filter_logits(logits: torch.Tensor, temperature: float = 1.0, top_k: int | None = None,
                  top_p: float | None = None) -> torch.Tensor:
    if temperature <= 0:
        raise ValueError("temperature must be > 0")
    logits = logits.float()
    if temperature != 1.0:
        logits = logits / temperature
    if top_k is not None and top_k > 0:
        kth = torch.topk(logits, k=min(top_k, logits.size(-1)), dim=-1).values[:, -1:]
        logits = logits.masked_fill(logits < kth, float("-inf"))
    if top_p is not None and 0 < top_p < 1.0:
        sorted_logits, order = torch.sort(logits, descending=True, dim=-1)
        cum = torch.softmax(sorted_logits, dim=-1).cumsum(dim=-1)
        drop = cum > top_p
        drop[..., 0] = False
        kept = sorted_logits.masked_fill(drop, float("-inf"))
        logits = torch.full_like(logits, float("-inf")).scatter_(-1, order, kept)
    return logits


def _cuda_sample(logits: torch.Tensor, temperature: float, top_k, top_p, with_log_prob: bool, generator=None,
                 rng: torch.Tensor | None = None, out=None):
    """One fused kernel (csrc/fused/sample.cu): temperature, top-k / top-p thresholds by
    radix selection, Philox draw.  The seed comes from a CPU generator (torch's global one
    unless ``generator`` is given), so ``set_seed`` makes sampling reproducible, ranks that
    share a generator state draw identical tokens, and no device sync is needed."""
    from tinytron_b200.ops import _ext

    if temperature <= 0:
        raise ValueError("temperature must be > 0")
    x = logits if logits.stride(-1) == 1 else logits.contiguous()
    if x.dtype not in (torch.bfloat16, torch.float32):
        x = x.float()
    B = x.shape[0]
    if out is not None:  # caller-owned outputs (a captured decode step)
        tok, lp = out
    else:
        tok = torch.empty(B, dtype=torch.long, device=x.device)
        lp = torch.empty(B, dtype=torch.float32, device=x.device) if with_log_prob else None
    # rng (device int64 [seed, offset]): the kernel reads the seed there, so a CUDA graph
    # replay draws fresh numbers; otherwise one seed per call from the CPU generator
    seed = 0 if rng is not None else int(torch.randint(0, 2 ** 62, (1,), generator=generator).item())
    _ext.load().sample_tokens(x, float(temperature), int(top_k or 0), float(top_p or 0.0), seed, 0, tok, lp, rng)
    return tok, lp


def sample_next_token(logits, temperature: float = 1.0, top_k=None, top_p=None, generator=None) -> torch.Tensor:
    if logits.is_cuda and logits.dim() == 2:
        return _cuda_sample(logits, temperature, top_k, top_p, False, generator)[0]
    if top_k == 1 and temperature > 0:  # greedy: identical result without a multinomial draw
        return logits.argmax(dim=-1)
    probs = torch.softmax(filter_logits(logits, temperature, top_k, top_p), dim=-1)
    return torch.multinomial(probs, num_samples=1, generator=generator).squeeze(-1)


def sample_next_token_with_log_prob(logits, temperature: float = 1.0, top_k=None, top_p=None, generator=None):
    if logits.is_cuda and logits.dim() == 2:
        return _cuda_sample(logits, temperature, top_k, top_p, True, generator)
    lp = torch.log_softmax(filter_logits(logits, temperature, top_k, top_p), dim=-1)
    tok = lp.argmax(dim=-1) if top_k == 1 else torch.multinomial(lp.exp(), num_samples=1,
                                                                  generator=generator).squeeze(-1)
    return tok, lp.gather(-1, tok.unsqueeze(-1)).squeeze(-1)
