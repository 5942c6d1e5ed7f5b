"""CPU fp32 parity of the framework's model against the reference model (same weights)."""
import pytest
import torch

import ref_oracle
from tinytron_b200.models import GPT, ModelConfig

pytestmark = pytest.mark.skipif(not ref_oracle.available(), reason="reference not installed under baseline/_ref")


def _cfgs():
    dense = ModelConfig(block_size=64, vocab_size=256, num_layer=2, num_attention_heads=4, num_key_value_heads=2,
                        hidden_size=64, intermediate_size=96, init_std=0.02, seed=7)
    moe = ModelConfig(block_size=64, vocab_size=256, num_layer=2, num_attention_heads=4, num_key_value_heads=2,
                      hidden_size=64, intermediate_size=96, init_std=0.02, seed=7, use_moe=True, num_experts=4,
                      num_experts_per_tok=2, moe_intermediate_size=48, moe_balance_loss_weight=0.01)
    return {"dense": dense, "moe": moe}


@pytest.fixture(scope="module")
def ref():
    ref_oracle.ensure_gloo_world1()
    with ref_oracle.cpu_reference() as tt:
        from tinytron.distributed import parallel_state
        from tinytron.training.config import ParallelConfig

        parallel_state.initialize_model_parallel(ParallelConfig(sep_size=1))
        yield tt


@pytest.mark.parametrize("kind", ["dense", "moe"])
def test_forward_backward_matches_reference(ref, kind):
    from tinytron.model import GPT as RefGPT
    from tinytron.model.config import ModelConfig as RefCfg

    cfg = _cfgs()[kind]
    ref_cfg = RefCfg(**{k: v for k, v in cfg.__dict__.items() if k in RefCfg.__dataclass_fields__})
    torch.manual_seed(0)
    rm = RefGPT(ref_cfg)
    ours = GPT(cfg, device="cpu")
    missing, unexpected = ours.load_state_dict(rm.state_dict(), strict=True)
    assert not missing and not unexpected
    x = torch.randint(0, cfg.vocab_size, (2, 32))
    y = torch.randint(0, cfg.vocab_size, (2, 32))
    y[0, :5] = -100
    _, rl, rll = rm(x, y)
    rl.backward()
    _, ol, oll = ours(x, y)
    ol.backward()
    assert torch.allclose(ol, rl, atol=1e-5, rtol=1e-5), (ol.item(), rl.item())
    assert torch.allclose(oll, rll, atol=1e-5, rtol=1e-5)
    rg = {n: p.grad for n, p in rm.named_parameters()}
    for n, p in ours.named_parameters():
        assert p.grad is not None, n
        assert torch.allclose(p.grad, rg[n], atol=1e-5, rtol=1e-4), n
    # logits path (no targets)
    assert torch.allclose(ours(x), rm(x), atol=1e-5, rtol=1e-5)
    # clip_grad_norm semantics
    assert torch.allclose(ours.clip_grad_norm(0.5), rm.clip_grad_norm(0.5), atol=1e-5, rtol=1e-5)


def test_kv_cache_decode_matches_reference(ref):
    from tinytron.model import GPT as RefGPT
    from tinytron.model.config import ModelConfig as RefCfg

    cfg = _cfgs()["dense"]
    rm = RefGPT(RefCfg(**{k: v for k, v in cfg.__dict__.items() if k in RefCfg.__dataclass_fields__})).eval()
    ours = GPT(cfg, device="cpu").eval()
    ours.load_state_dict(rm.state_dict())
    x = torch.randint(0, cfg.vocab_size, (2, 10))
    with torch.no_grad():
        rl, rkv = rm(x, use_cache=True)
        ol, okv = ours(x, use_cache=True)
        assert torch.allclose(ol, rl, atol=1e-5)
        nxt = torch.randint(0, cfg.vocab_size, (2, 1))
        rl2, _ = rm(nxt, use_cache=True, past_key_values=rkv, position_offset=10)
        ol2, _ = ours(nxt, use_cache=True, past_key_values=okv, position_offset=10)
        assert torch.allclose(ol2, rl2, atol=1e-5)


@pytest.mark.parametrize("paged", [True, False])
def test_engine_generate_matches_reference(ref, paged):
    """InferenceEngine.generate on CPU in fp32, same weights: greedy tokens, their
    log-probs and the EOS stop agree with the reference engine."""
    from tinytron.inference import InferenceEngine as RefEngine
    from tinytron.model.config import ModelConfig as RefCfg

    from tinytron_b200.inference import InferenceEngine

    cfg = _cfgs()["moe"]
    rcfg = RefCfg(**{k: v for k, v in cfg.__dict__.items() if k in RefCfg.__dataclass_fields__})
    torch.manual_seed(0)
    re = RefEngine(rcfg, device="cpu", dtype=torch.float32, use_paged_kv_cache=paged, kv_cache_page_size=4)
    oe = InferenceEngine(cfg, device="cpu", dtype=torch.float32, use_paged_kv_cache=paged, kv_cache_page_size=4)
    oe.model.load_state_dict(re.model.state_dict())
    prompt = torch.randint(0, cfg.vocab_size, (3, 9), generator=torch.Generator().manual_seed(2))
    rt, rinfo = re.generate(prompt, 12, temperature=1.0, top_k=1, return_logprobs=True)
    ot, oinfo = oe.generate(prompt, 12, temperature=1.0, top_k=1, return_logprobs=True)
    assert torch.equal(ot.cpu(), rt.cpu())
    assert torch.allclose(oinfo["token_log_probs"].cpu(), rinfo["token_log_probs"].cpu(), atol=1e-5)
    eos = int(rt[0, 9 + 4])  # stop when sequence 0 emits its 5th generated token
    rt2 = re.generate(prompt, 12, temperature=1.0, top_k=1, eos_token_id=eos)
    ot2 = oe.generate(prompt, 12, temperature=1.0, top_k=1, eos_token_id=eos)
    assert torch.equal(ot2.cpu(), rt2.cpu())


def test_engine_extras_match_reference(ref):
    """generate(..., return_stats=True, return_logprobs=True) returns the reference's extra
    keys; the counts (prompt length, decode steps, token counts) and the response mask
    agree, the throughput fields are positive."""
    from tinytron.inference import InferenceEngine as RefEngine
    from tinytron.model.config import ModelConfig as RefCfg

    from tinytron_b200.inference import InferenceEngine

    cfg = _cfgs()["dense"]
    rcfg = RefCfg(**{k: v for k, v in cfg.__dict__.items() if k in RefCfg.__dataclass_fields__})
    torch.manual_seed(0)
    re = RefEngine(rcfg, device="cpu", dtype=torch.float32, use_paged_kv_cache=True, kv_cache_page_size=4)
    oe = InferenceEngine(cfg, device="cpu", dtype=torch.float32, use_paged_kv_cache=True, kv_cache_page_size=4)
    oe.model.load_state_dict(re.model.state_dict())
    prompt = torch.randint(0, cfg.vocab_size, (2, 6), generator=torch.Generator().manual_seed(5))
    for n_new in (1, 5):
        _, r = re.generate(prompt, n_new, top_k=1, return_stats=True, return_logprobs=True)
        _, o = oe.generate(prompt, n_new, top_k=1, return_stats=True, return_logprobs=True)
        assert set(r) <= set(o), sorted(set(r) - set(o))
        for k in ("prompt_len", "decode_steps", "prefill_tokens", "decode_tokens"):
            assert float(o[k]) == float(r[k]), (n_new, k, o[k], r[k])
        assert torch.equal(o["response_mask"].cpu(), r["response_mask"].cpu())
        assert o["prefill_tokens_per_sec"] > 0 and (o["decode_tokens_per_sec"] > 0) == (r["decode_tokens_per_sec"] > 0)
