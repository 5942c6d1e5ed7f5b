"""Inference entry point (reference: scripts/debug/inference.py:21-128).

    python -m tinytron_b200.launch.inference --init_from_scratch --prompt_token_ids 1,2,3 --max_new_tokens 16
    torchrun --nproc-per-node 8 -m tinytron_b200.launch.inference --checkpoint_path <..._model.pt> --sep_size 8

With ``--batch_size B --prompt_len P`` (instead of ``--prompt_token_ids``) it runs a
synthetic batch of seeded uniform prompts and prints prefill/decode tokens per second.
"""
from __future__ import annotations

import os
from dataclasses import replace

import torch
import torch.distributed as dist

from tinytron_b200.inference import InferenceEngine
from tinytron_b200.inference.arguments import build_parser, parse_prompt_token_ids
from tinytron_b200.inference.checkpoint import checkpoint_meta_path, checkpoint_prefix_from_model_path
from tinytron_b200.models.config import ModelConfig, build_model_config
from tinytron_b200.parallel import parallel_state
from tinytron_b200.training.config import ParallelConfig

from ._presets import expand_preset


def _distributed() -> bool:
    return int(os.environ.get("WORLD_SIZE", "1")) > 1


def _init(args) -> tuple[str, bool]:
    if not _distributed():
        return args.device, True
    dist.init_process_group(backend=args.backend, init_method=args.init_method)
    local = int(os.environ["LOCAL_RANK"])
    if args.device not in ("cuda", f"cuda:{local}"):
        raise ValueError(f"distributed inference rank {local} must use device cuda:{local}; got {args.device!r}")
    torch.cuda.set_device(local)
    parallel_state.initialize_model_parallel(ParallelConfig(backend=args.backend, init_method=args.init_method,
                                                            sep_size=args.sep_size))
    return f"cuda:{local}", dist.get_rank() == 0


def _model_config(args) -> ModelConfig:
    cfg_dict = None
    if args.checkpoint_path:
        prefix = checkpoint_prefix_from_model_path(args.checkpoint_path)
        meta = checkpoint_meta_path(prefix) if prefix is not None else None
        if meta is not None and os.path.exists(meta):
            cfg_dict = torch.load(meta, map_location="cpu", weights_only=False).get("config", {}).get("model")
    cfg = build_model_config(args, seed=args.seed) if cfg_dict is None else ModelConfig(**cfg_dict)
    if args.inference_shard_qkv is not None:
        cfg = replace(cfg, inference_shard_qkv=args.inference_shard_qkv)
    return cfg


def main(argv: list[str] | None = None) -> None:
    parser = build_parser()
    parser.add_argument("--batch_size", type=int, default=0, help="synthetic prompts (with --prompt_len)")
    parser.add_argument("--prompt_len", type=int, default=0)
    parser.add_argument("--no_cuda_graph", action="store_true", help="decode eagerly instead of graph replay")
    args = parser.parse_args(expand_preset(argv))
    if not args.init_from_scratch and not args.checkpoint_path:
        parser.error("Either provide --checkpoint_path, or set --init_from_scratch for random-weight smoke testing.")
    if _distributed() and args.sep_size <= 1:
        parser.error("Distributed inference requires --sep_size > 1 to initialize SEP process groups.")
    cfg = _model_config(args)
    try:
        device, master = _init(args)
        dtype = torch.bfloat16 if args.dtype == "bf16" else torch.float32
        if args.batch_size > 0 and args.prompt_len > 0:
            g = torch.Generator().manual_seed(args.seed)
            prompt = torch.randint(0, cfg.vocab_size, (args.batch_size, args.prompt_len), generator=g)
        else:
            prompt = torch.tensor([parse_prompt_token_ids(args.prompt_token_ids)], dtype=torch.long)
        engine = InferenceEngine(model_config=cfg, checkpoint_path=args.checkpoint_path, device=device, dtype=dtype,
                                 use_paged_kv_cache=args.paged_kv_cache, kv_cache_page_size=args.kv_cache_page_size,
                                 use_cuda_graph=not args.no_cuda_graph)
        out, stats = engine.generate(prompt, max_new_tokens=args.max_new_tokens, temperature=args.temperature,
                                     top_k=args.top_k, top_p=args.top_p, eos_token_id=args.eos_token_id,
                                     return_stats=True)
        if master:
            if prompt.shape[0] == 1:
                print(",".join(str(int(x)) for x in out[0].tolist()))
            print(f"prefill tok/s: {stats['prefill_tokens_per_sec']:.2f}")
            print(f"decode tok/s: {stats['decode_tokens_per_sec']:.2f}")
    finally:
        if dist.is_available() and dist.is_initialized():
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
