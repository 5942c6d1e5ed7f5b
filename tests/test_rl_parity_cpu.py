"""RL primitives against the reference's on the same inputs (CPU, no process group):
log-prob helpers, masked reductions, response masks, rollout batches, group advantages
and the policy-gradient / PPO / GRPO / DPO losses with their metrics.  Skipped when the
reference is not installed under baseline/_ref."""
import pytest
import torch

from ref_oracle import available, cpu_reference

pytestmark = pytest.mark.skipif(not available(), reason="reference not installed under baseline/_ref")


@pytest.fixture(scope="module")
def ref_rl():
    with cpu_reference():
        import tinytron.rl as rl

        yield rl


def _close(a, b, tol=1e-6):
    if isinstance(a, torch.Tensor) or isinstance(b, torch.Tensor):
        a, b = torch.as_tensor(a).float(), torch.as_tensor(b).float()
        return a.shape == b.shape and torch.allclose(a, b, atol=tol, rtol=tol)
    return a == b


def _same_output(o, r):
    assert _close(o.loss, r.loss), (o.loss, r.loss)
    assert set(o.metrics) == set(r.metrics), (sorted(o.metrics), sorted(r.metrics))
    for k in r.metrics:
        assert _close(o.metrics[k], r.metrics[k]), (k, o.metrics[k], r.metrics[k])


def test_log_prob_helpers_match(ref_rl):
    import tinytron_b200.rl as rl

    g = torch.Generator().manual_seed(0)
    logits = torch.randn(3, 7, 11, generator=g)
    seq = torch.randint(0, 11, (3, 7), generator=g)
    assert _close(rl.gather_log_probs(logits, seq), ref_rl.gather_log_probs(logits, seq))
    assert _close(rl.causal_log_probs(logits, seq), ref_rl.causal_log_probs(logits, seq))
    mask = torch.rand(3, 6, generator=g) > 0.4
    assert _close(rl.response_log_probs(logits, seq, mask), ref_rl.response_log_probs(logits, seq, mask))
    vals = torch.randn(3, 6, generator=g)
    for m in (mask, mask.float(), torch.zeros_like(mask)):
        assert _close(rl.masked_sum(vals, m), ref_rl.masked_sum(vals, m))
        assert _close(rl.masked_mean(vals, m), ref_rl.masked_mean(vals, m))
        for avg in (False, True):
            assert _close(rl.sequence_log_probs(vals, m, average=avg), ref_rl.sequence_log_probs(vals, m, average=avg))


@pytest.mark.parametrize("eos", [None, 3])
def test_response_mask_and_rollout_batch_match(ref_rl, eos):
    import tinytron_b200.rl as rl

    g = torch.Generator().manual_seed(1)
    prompts = torch.randint(4, 11, (4, 5), generator=g)
    resp = torch.randint(0, 11, (4, 8), generator=g)
    resp[1, 2] = 3  # an EOS inside one response
    resp[2, 0] = 3  # and as the first response token
    seq = torch.cat([prompts, resp], 1)
    assert torch.equal(rl.build_response_mask(seq, 5, eos), ref_rl.build_response_mask(seq, 5, eos))
    old = torch.randn(4, 8, generator=g)  # the sampler's log-probs of the 8 generated tokens
    for bad in (torch.randn(4, 12), torch.randn(3, 8)):  # both reject misaligned log-probs
        with pytest.raises(ValueError):
            rl.make_rollout_batch(prompts, seq, old_log_probs=bad, eos_token_id=eos)
        with pytest.raises(ValueError):
            ref_rl.make_rollout_batch(prompts, seq, old_log_probs=bad, eos_token_id=eos)
    ob = rl.make_rollout_batch(prompts, seq, old_log_probs=old, eos_token_id=eos)
    rb = ref_rl.make_rollout_batch(prompts, seq, old_log_probs=old, eos_token_id=eos)
    for f in ("prompts", "responses", "sequences", "labels", "response_mask", "prompt_lens", "response_lens",
              "old_log_probs", "reference_log_probs"):
        a, b = getattr(ob, f), getattr(rb, f)
        assert (a is None and b is None) or (a is not None and b is not None and _close(a, b)), f


def test_group_advantages_match(ref_rl):
    import tinytron_b200.rl as rl

    g = torch.Generator().manual_seed(2)
    rewards = torch.randn(12, generator=g)
    for gs in (1, 3, 4, 12):
        assert _close(rl.group_advantages(rewards, gs), ref_rl.group_advantages(rewards, gs)), gs
    flat = torch.ones(8)  # zero variance inside every group
    assert _close(rl.group_advantages(flat, 4), ref_rl.group_advantages(flat, 4))


@pytest.mark.parametrize("adv_shape", ["token", "sequence"])
def test_losses_match(ref_rl, adv_shape):
    import tinytron_b200.rl as rl

    g = torch.Generator().manual_seed(3)
    B, T = 4, 9
    lp = torch.randn(B, T, generator=g) * 0.3 - 1
    old = lp + torch.randn(B, T, generator=g) * 0.2
    refp = lp + torch.randn(B, T, generator=g) * 0.1
    mask = torch.rand(B, T, generator=g) > 0.3
    adv = torch.randn(B, T, generator=g) if adv_shape == "token" else torch.randn(B, generator=g)
    _same_output(rl.policy_gradient_loss(lp, adv, mask), ref_rl.policy_gradient_loss(lp, adv, mask))
    for clip in (0.1, 0.2):
        _same_output(rl.ppo_policy_loss(lp, old, adv, mask, clip_range=clip),
                     ref_rl.ppo_policy_loss(lp, old, adv, mask, clip_range=clip))
    for rp, kl in ((None, 0.0), (refp, 0.0), (refp, 0.05)):
        _same_output(rl.grpo_loss(lp, old, adv, mask, reference_log_probs=rp, clip_range=0.2, kl_coef=kl),
                     ref_rl.grpo_loss(lp, old, adv, mask, reference_log_probs=rp, clip_range=0.2, kl_coef=kl))
    assert _close(rl.approx_kl(lp, refp, mask), ref_rl.approx_kl(lp, refp, mask))
    c, r, rc, rr = (torch.randn(B, generator=g) for _ in range(4))
    for beta in (0.1, 0.5):
        _same_output(rl.dpo_loss(c, r, rc, rr, beta=beta), ref_rl.dpo_loss(c, r, rc, rr, beta=beta))


def test_rl_config_and_sync_helpers_match(ref_rl):
    """RLConfig keeps the reference's fields and defaults; inference_model_config and
    unwrap_model behave the same; the actor -> rollout state dict at SEP=1 holds the same
    tensors."""
    import dataclasses

    import torch.nn as nn

    import ref_oracle
    import tinytron_b200.rl as rl
    from tinytron_b200.models import GPT, ModelConfig

    ref_fields = {f.name: f.default for f in dataclasses.fields(ref_rl.RLConfig)}
    our_fields = {f.name: f.default for f in dataclasses.fields(rl.RLConfig)}
    for k, v in ref_fields.items():
        assert k in our_fields and our_fields[k] == v, (k, our_fields.get(k), v)
    cfg = ModelConfig(block_size=32, vocab_size=64, num_layer=1, num_attention_heads=4, num_key_value_heads=2,
                      hidden_size=32, intermediate_size=48)
    with cpu_reference():
        from tinytron.model.config import ModelConfig as RefCfg

        rcfg = RefCfg(**{k: v for k, v in cfg.__dict__.items() if k in RefCfg.__dataclass_fields__})
    for shard in (True, False):
        assert rl.inference_model_config(cfg, shard).inference_shard_qkv == \
            ref_rl.inference_model_config(rcfg, shard).inference_shard_qkv == shard
    m = nn.Linear(2, 2)
    wrapped = nn.Module()
    wrapped.module = m
    assert rl.unwrap_model(wrapped) is m and ref_rl.unwrap_model(wrapped) is m and rl.unwrap_model(m) is m
    ref_oracle.ensure_gloo_world1(port=29617)
    model = GPT(cfg, device="cpu")
    ours = rl.training_state_dict_to_inference(model, rl.inference_model_config(cfg, False))
    with cpu_reference():
        from tinytron.distributed import parallel_state
        from tinytron.training.config import ParallelConfig

        parallel_state.initialize_model_parallel(ParallelConfig(sep_size=1))
        theirs = ref_rl.training_state_dict_to_inference(model, ref_rl.inference_model_config(rcfg, False))
    assert set(ours) == set(theirs)
    for k in theirs:
        assert torch.equal(ours[k].cpu(), theirs[k].cpu()), k
