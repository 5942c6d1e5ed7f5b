"""Paged decode kernels (fused RoPE + KV append, split-KV attention) and the
CUDA-graph decode engine vs plain PyTorch fp32 references."""
import math

import pytest
import torch

pytestmark = pytest.mark.gpu


def ext():
    from tinytron_b200.ops import _ext

    return _ext.load()


def _pages(B, L, Hkv, D, page_size, gen):
    pps = math.ceil(L / page_size)
    num_pages = B * pps + 3
    perm = torch.randperm(num_pages, generator=gen)[: B * pps].view(B, pps).to(torch.int32)
    k_pages = torch.randn(num_pages, page_size, Hkv, D, generator=gen).bfloat16()
    v_pages = torch.randn(num_pages, page_size, Hkv, D, generator=gen).bfloat16()
    return perm, k_pages, v_pages


def _gather(pages, table, L):
    B, pps = table.shape
    P = pages.shape[1]
    x = pages[table.long()].reshape(B, pps * P, pages.shape[2], pages.shape[3])
    return x[:, :L]  # [B, L, Hkv, D]


@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("G", [1, 2, 4, 8])
@pytest.mark.parametrize("L,page_size", [(1, 16), (17, 16), (256, 16), (257, 16), (1000, 16), (700, 700)])
def test_decode_attention_matches_fp32(D, G, L, page_size):
    gen = torch.Generator().manual_seed(L * 7 + G)
    B, Hkv = 3, 2
    Hq = Hkv * G
    table, kp, vp = _pages(B, L, Hkv, D, page_size, gen)
    q = torch.randn(B, Hq, D, generator=gen).bfloat16()
    C = ext()
    splits = int(C.decode_num_splits(L + 40))  # more splits than needed: empty ones must be ignored
    o_part = torch.empty(B * Hq * splits * D, device="cuda")
    ml = torch.empty(B * Hq * splits * 2, device="cuda")
    out = torch.empty(B, Hq * D, device="cuda", dtype=torch.bfloat16)
    len_dev = torch.tensor([L - 1], dtype=torch.int32, device="cuda")
    scale = 1 / math.sqrt(D)
    C.decode_attention(q.cuda(), kp.cuda(), vp.cuda(), table.cuda(), len_dev, 1, splits, scale, o_part, ml, out)
    torch.cuda.synchronize()
    k = _gather(kp, table, L).float()
    v = _gather(vp, table, L).float()
    kq = k.repeat_interleave(G, dim=2)  # [B, L, Hq, D]
    vq = v.repeat_interleave(G, dim=2)
    s = torch.einsum("bhd,blhd->bhl", q.float(), kq) * scale
    ref = torch.einsum("bhl,blhd->bhd", s.softmax(-1), vq).reshape(B, Hq * D)
    err = (out.float().cpu() - ref).abs().max().item()
    assert err < 2e-2, err


@pytest.mark.parametrize("T,pos0", [(1, 0), (1, 37), (5, 16), (33, 100)])
def test_rope_append_matches_reference(T, pos0):
    from tinytron_b200.ops.rope import rope_reference, rope_tables

    gen = torch.Generator().manual_seed(T + pos0)
    B, Hq, Hkv, D, P = 2, 4, 2, 128, 16
    L = pos0 + T
    table, kp, vp = _pages(B, L, Hkv, D, P, gen)
    kp, vp, table = kp.cuda(), vp.cuda(), table.cuda()
    qkv = torch.randn(B * T, (Hq + 2 * Hkv) * D, generator=gen).bfloat16().cuda()
    cos, sin = rope_tables(D, 10000.0, 4096, "cuda")
    q_out = torch.empty(B * T, Hq * D, dtype=torch.bfloat16, device="cuda")
    pos_dev = torch.tensor([pos0], dtype=torch.int32, device="cuda")
    ext().decode_rope_append(qkv, B, T, Hq, Hkv, D, pos_dev, 0, cos, sin, q_out, kp, vp, table)
    torch.cuda.synchronize()
    x = qkv.float().view(B, T, Hq + 2 * Hkv, D).transpose(1, 2)
    pos = torch.arange(pos0, pos0 + T, device="cuda")
    qr, kr = rope_reference(x[:, :Hq], x[:, Hq:Hq + Hkv], pos)
    assert (q_out.float().view(B, T, Hq, D).transpose(1, 2) - qr).abs().max().item() < 3e-2
    kc = _gather(kp, table, L)[:, pos0:].float().transpose(1, 2)  # [B, Hkv, T, D]
    vc = _gather(vp, table, L)[:, pos0:].float().transpose(1, 2)
    assert (kc - kr).abs().max().item() < 3e-2
    assert torch.equal(vc, x[:, Hq + Hkv:].bfloat16().float())


def _tiny_cfg(**kw):
    from tinytron_b200.models import ModelConfig

    base = dict(block_size=512, vocab_size=512, num_layer=2, num_attention_heads=8, num_key_value_heads=2,
                hidden_size=512, intermediate_size=1024, init_std=0.02, seed=5)
    base.update(kw)
    return ModelConfig(**base)


@pytest.mark.parametrize("paged", [True, False])
def test_engine_graph_decode_matches_eager_and_cpu(paged):
    from tinytron_b200.inference import InferenceEngine

    cfg = _tiny_cfg()
    eng_g = InferenceEngine(cfg, device="cuda", use_paged_kv_cache=paged, kv_cache_page_size=16, use_cuda_graph=True)
    eng_e = InferenceEngine(cfg, device="cuda", use_paged_kv_cache=paged, kv_cache_page_size=16,
                            use_cuda_graph=False)
    eng_e.model.load_state_dict(eng_g.model.state_dict())
    prompt = torch.randint(0, cfg.vocab_size, (4, 40), generator=torch.Generator().manual_seed(0))
    tg = eng_g.generate(prompt, 24, temperature=1.0, top_k=1)
    te = eng_e.generate(prompt, 24, temperature=1.0, top_k=1)
    assert torch.equal(tg.cpu(), te.cpu())
    # step logits of the fused cached path vs the fp32 CPU model on the full sequence
    cpu = eng_g.model.__class__(cfg, device="cpu")
    cpu.load_state_dict({k: v.cpu() for k, v in eng_g.model.state_dict().items()})
    cpu.eval()
    with torch.no_grad():
        ref = cpu(tg.cpu())  # [B, T, V] logits (no targets)
        ref = ref[0] if isinstance(ref, tuple) else ref
        cache = eng_e.new_cache(4, max_seq_len=tg.shape[1])
        cache.reserve(tg.shape[1])
        n = 40
        logits, cache = eng_e.model._forward_cached(tg[:, :n].cuda(), cache, True, 0, last_only=True)
        errs = [(logits[:, -1].float().cpu() - ref[:, n - 1]).abs().max().item()]
        for t in range(n, tg.shape[1] - 1):
            logits, cache = eng_e.model._forward_cached(tg[:, t:t + 1].cuda(), cache, True, t, last_only=True)
            errs.append((logits[:, -1].float().cpu() - ref[:, t]).abs().max().item())
    scale = ref.abs().max().item()
    assert max(errs) < 3e-2 * scale + 2e-2, (max(errs), scale)


def test_engine_graph_decode_moe():
    from tinytron_b200.inference import InferenceEngine

    cfg = _tiny_cfg(use_moe=True, num_experts=8, num_experts_per_tok=2, moe_intermediate_size=256)
    eng_g = InferenceEngine(cfg, device="cuda", kv_cache_page_size=16, use_cuda_graph=True)
    eng_e = InferenceEngine(cfg, device="cuda", kv_cache_page_size=16, use_cuda_graph=False)
    eng_e.model.load_state_dict(eng_g.model.state_dict())
    prompt = torch.randint(0, cfg.vocab_size, (2, 24), generator=torch.Generator().manual_seed(1))
    tg, sg = eng_g.generate(prompt, 12, temperature=1.0, top_k=1, return_stats=True)
    te = eng_e.generate(prompt, 12, temperature=1.0, top_k=1)
    assert torch.equal(tg.cpu(), te.cpu())
    assert sg["decode_tokens_per_sec"] > 0


def test_engine_graph_sampling_is_reproducible_and_valid():
    """Temperature/top-k draws inside the captured decode step: the seed and Philox offset
    live on the device, so every replay draws fresh numbers, and a seeded run repeats."""
    from tinytron_b200.inference import InferenceEngine

    cfg = _tiny_cfg()
    eng = InferenceEngine(cfg, device="cuda", kv_cache_page_size=16, use_cuda_graph=True)
    prompt = torch.randint(0, cfg.vocab_size, (4, 20), generator=torch.Generator().manual_seed(2))
    runs = []
    for _ in range(2):
        torch.manual_seed(5)
        toks, info = eng.generate(prompt, 16, temperature=1.0, top_k=50, return_logprobs=True)
        runs.append((toks.cpu(), info["token_log_probs"].cpu()))
    assert torch.equal(runs[0][0], runs[1][0]) and torch.equal(runs[0][1], runs[1][1])
    toks, lp = runs[0]
    assert toks.shape == (4, 36) and lp.shape == (4, 16)
    assert torch.equal(toks[:, :20], prompt)
    assert bool(((toks >= 0) & (toks < cfg.vocab_size)).all())
    assert bool(torch.isfinite(lp).all()) and bool((lp <= 0).all())
    # fresh draws per step: a random-init model at temperature 1 does not repeat one token
    assert len(set(toks[:, 20:].reshape(-1).tolist())) > 8
    torch.manual_seed(6)
    other = eng.generate(prompt, 16, temperature=1.0, top_k=50).cpu()
    assert not torch.equal(other, toks)
