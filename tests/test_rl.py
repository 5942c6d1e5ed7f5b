"""RL primitives (semantics of the reference's tests/test_rl.py, plus GRPO/KL checks)."""
import torch

from tinytron_b200.rl import (build_response_mask, dpo_loss, gather_log_probs, group_advantages, grpo_loss,
                              make_rollout_batch, ppo_policy_loss, sequence_log_probs)


def test_gather_log_probs():
    logits = torch.tensor([[[1.0, 2.0, 3.0], [3.0, 0.0, 1.0]]])
    ids = torch.tensor([[2, 0]])
    want = torch.log_softmax(logits, -1).gather(-1, ids.unsqueeze(-1)).squeeze(-1)
    assert torch.allclose(gather_log_probs(logits, ids), want)


def test_response_mask_eos():
    seq = torch.tensor([[1, 2, 3, 4, 5], [1, 2, 9, 8, 7]])
    m = build_response_mask(seq, prompt_len=2, eos_token_id=4)
    assert torch.equal(m, torch.tensor([[0.0, 1.0, 1.0, 0.0], [0.0, 1.0, 1.0, 1.0]]))


def test_sequence_log_probs():
    lp = torch.tensor([[-1.0, -2.0, -3.0], [-4.0, -5.0, -6.0]])
    m = torch.tensor([[1.0, 0.0, 1.0], [0.0, 1.0, 1.0]])
    assert torch.allclose(sequence_log_probs(lp, m), torch.tensor([-4.0, -11.0]))
    assert torch.allclose(sequence_log_probs(lp, m, average=True), torch.tensor([-2.0, -5.5]))


def test_rollout_batch_labels_and_masks():
    prompts = torch.tensor([[1, 2], [3, 4]])
    seqs = torch.tensor([[1, 2, 5, 6], [3, 4, 7, 0]])
    old = torch.tensor([[-0.1, -0.2], [-0.3, -0.4]])
    b = make_rollout_batch(prompts, seqs, old_log_probs=old, eos_token_id=7)
    assert torch.equal(b.labels, torch.tensor([[-100, 5, 6], [-100, 7, -100]]))
    assert torch.equal(b.response_mask, torch.tensor([[0.0, 1.0, 1.0], [0.0, 1.0, 0.0]]))
    assert torch.equal(b.response_lens, torch.tensor([2, 1]))
    assert torch.allclose(b.old_log_probs, torch.tensor([[0.0, -0.1, -0.2], [0.0, -0.3, -0.4]]))


def test_dpo_prefers_chosen():
    good = dpo_loss(torch.tensor([0.0]), torch.tensor([-2.0]), torch.tensor([-1.0]), torch.tensor([-1.0]))
    bad = dpo_loss(torch.tensor([-2.0]), torch.tensor([0.0]), torch.tensor([-1.0]), torch.tensor([-1.0]))
    assert good.loss < bad.loss and good.metrics["reward_accuracy"].item() == 1.0


def test_ppo_accepts_sequence_advantages():
    lp = torch.zeros(2, 3, requires_grad=True)
    out = ppo_policy_loss(lp, torch.zeros(2, 3), torch.tensor([1.0, -1.0]), torch.ones(2, 3))
    out.loss.backward()
    assert lp.grad is not None and torch.isfinite(out.loss)


def test_group_advantages_and_grpo_kl():
    adv = group_advantages(torch.tensor([1.0, 3.0, 0.0, 0.0]), 2)
    assert torch.allclose(adv, torch.tensor([-1.0, 1.0, 0.0, 0.0]))
    lp = torch.tensor([[-1.0, -1.0]])
    out = grpo_loss(lp, lp, torch.tensor([1.0]), torch.ones(1, 2), reference_log_probs=lp - 0.5, kl_coef=0.1)
    assert out.metrics["kl"].item() > 0


def test_sampler_filter_matches_reference():
    import pytest as _pytest
    import ref_oracle

    if not ref_oracle.available():
        _pytest.skip("reference not installed under baseline/_ref")
    from tinytron_b200.inference.sampler import filter_logits, sample_next_token_with_log_prob

    with ref_oracle.cpu_reference():
        from tinytron.inference.sampler import filter_logits as ref_filter
        from tinytron.inference.sampler import sample_next_token_with_log_prob as ref_sample_lp
    g = torch.Generator().manual_seed(0)
    logits = torch.randn(6, 300, generator=g) * 3
    for t, k, p in [(1.0, None, None), (0.7, 20, None), (1.3, None, 0.8), (0.9, 50, 0.6), (1.0, 1, None)]:
        assert torch.equal(filter_logits(logits, t, k, p), ref_filter(logits, t, k, p)), (t, k, p)
        torch.manual_seed(5)
        ours = sample_next_token_with_log_prob(logits, t, k, p)
        torch.manual_seed(5)
        ref = ref_sample_lp(logits, t, k, p)
        assert torch.equal(ours[0], ref[0]) and torch.allclose(ours[1], ref[1]), (t, k, p)
