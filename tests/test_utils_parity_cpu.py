"""The `utils` helpers return what the reference's return for the same inputs: training
budget (gradient accumulation, steps, epochs, and the error when budgets disagree),
parameter counts of dense and MoE configs, and the compiled -> uncompiled checkpoint
key mapping.  Skipped when the reference is not installed under baseline/_ref."""
import pytest
import torch

from ref_oracle import available, cpu_reference

pytestmark = pytest.mark.skipif(not available(), reason="reference not installed under baseline/_ref")


@pytest.mark.parametrize("kw", [
    dict(num_samples=1000, tokens_per_sample=4096, global_token_batch_size=524288,
         samples_per_dp_rank_per_micro_step=4, dp_world_size=8, max_steps=100),
    dict(num_samples=5000, tokens_per_sample=1024, global_token_batch_size=65536,
         samples_per_dp_rank_per_micro_step=2, dp_world_size=4, max_epochs=3),
    dict(num_samples=64, tokens_per_sample=128, global_token_batch_size=2048,
         samples_per_dp_rank_per_micro_step=1, dp_world_size=2, max_steps=16, max_epochs=4),
])
def test_training_info_matches_reference(kw):
    with cpu_reference():
        from tinytron.utils import get_training_info as ref_fn
    from tinytron_b200.utils import get_training_info

    assert get_training_info(**kw) == ref_fn(**kw)


def test_training_info_rejects_the_same_inputs():
    with cpu_reference():
        from tinytron.utils import get_training_info as ref_fn
    from tinytron_b200.utils import get_training_info

    for kw in (dict(num_samples=64, tokens_per_sample=128, global_token_batch_size=2048,
                    samples_per_dp_rank_per_micro_step=1, dp_world_size=2, max_steps=16, max_epochs=9),
               dict(num_samples=64, tokens_per_sample=128, global_token_batch_size=2048,
                    samples_per_dp_rank_per_micro_step=1, dp_world_size=2)):
        with pytest.raises(ValueError):
            ref_fn(**kw)
        with pytest.raises(ValueError):
            get_training_info(**kw)


@pytest.mark.parametrize("moe", [False, True])
def test_model_params_match_reference(moe):
    kw = dict(block_size=4096, vocab_size=50304, num_layer=24, num_attention_heads=16, num_key_value_heads=4,
              hidden_size=2048, intermediate_size=5504)
    if moe:
        kw.update(use_moe=True, num_experts=64, num_experts_per_tok=8, moe_intermediate_size=1408)
    with cpu_reference():
        from tinytron.model import ModelConfig as RefConfig
        from tinytron.utils import get_model_params as ref_fn

        ref = ref_fn(RefConfig(**kw))
    from tinytron_b200.models import ModelConfig
    from tinytron_b200.utils import get_model_params

    assert get_model_params(ModelConfig(**kw)) == pytest.approx(ref)


def test_compiled_key_mapping_matches_reference(capsys):
    from tinytron_b200.models import GPT, ModelConfig
    from tinytron_b200.utils import get_compiled_to_uncompiled_mapping

    c = ModelConfig(block_size=32, vocab_size=64, num_layer=1, num_attention_heads=2, num_key_value_heads=1,
                    hidden_size=32, intermediate_size=48)
    m = GPT(c, device="cpu")
    keys = ["_orig_mod." + k for k in list(m.state_dict())[:3]] + [list(m.state_dict())[3], "_orig_mod.not_a_key"]
    with cpu_reference():
        from tinytron.utils import get_compiled_to_uncompiled_mapping as ref_fn

        ref = ref_fn(m, keys)
    ours = get_compiled_to_uncompiled_mapping(m, keys)
    assert set(ours) == set(ref)
    for k in ref:
        assert torch.equal(ours[k], ref[k])


@pytest.mark.parametrize("path", ["ckpt/model_step_100.pt", "ckpt/model_step_100_rank0.pt", "a/b/c.pt",
                                  "ckpt/model_step_7_meta.pt", "ckpt/model_step_7", "", "/abs/x_model.pt",
                                  "ckpt/step_3_model_rank12.pt"])
def test_inference_checkpoint_paths_match_reference(path):
    with cpu_reference():
        from tinytron.inference import checkpoint as ref
    from tinytron_b200.inference import checkpoint as ours

    assert ours.checkpoint_prefix_from_model_path(path) == ref.checkpoint_prefix_from_model_path(path)
    prefix = "ckpt/model_step_5"
    assert ours.checkpoint_meta_path(prefix) == ref.checkpoint_meta_path(prefix)
    for r in (0, 3, 15):
        assert ours.checkpoint_model_shard_path(prefix, r) == ref.checkpoint_model_shard_path(prefix, r)


@pytest.mark.parametrize("gpu", ["NVIDIA H100 80GB HBM3", "NVIDIA A100-SXM4-80GB", "NVIDIA L40S", "Tesla V100"])
def test_peak_flops_and_mfu_match_reference(monkeypatch, gpu):
    """With the device name faked: the same peak for every dtype and both per-device
    modes, and compute_mfu's (mfu, achieved, peak) for the same model FLOP count."""
    monkeypatch.setattr(torch.cuda, "is_available", lambda: True)
    monkeypatch.setattr(torch.cuda, "get_device_name", lambda *a, **k: gpu)
    monkeypatch.setattr(torch.cuda, "device_count", lambda: 8)
    with cpu_reference():
        from tinytron.utils import compute_mfu as ref_mfu
        from tinytron.utils import get_gpu_peak_flops as ref_peak
    from tinytron_b200.utils import compute_mfu, get_gpu_peak_flops

    for dtype in ("bf16", "fp16", "fp32", "BF16"):
        for per_device in (True, False):
            assert get_gpu_peak_flops(dtype, per_device) == ref_peak(dtype, per_device), (dtype, per_device)

    class _Model:
        def get_flops_per_fwd_bwd(self, batch_size, seq_len):
            return 6.0 * 1.3e9 * batch_size * seq_len

    for ga in (1, 4):
        assert compute_mfu(_Model(), 4, 4096, 0.6, ga=ga) == pytest.approx(ref_mfu(_Model(), 4, 4096, 0.6, ga=ga))


@pytest.mark.parametrize("parts,ranks_map", [(1, None), (3, None), (4, None), (None, [5, 1, 3])])
def test_partition_tensors_matches_reference(parts, ranks_map):
    """The ZeRO-1 whole-tensor partition (largest first onto the least-loaded part, ties by
    key) assigns every tensor to the same part as the reference's."""
    from collections import OrderedDict

    from tinytron_b200.parallel.zero1 import partition_tensors

    g = torch.Generator().manual_seed(4)
    sizes = [int(x) for x in torch.randint(1, 50, (23,), generator=g)] + [7, 7, 7, 7]  # with ties
    td = OrderedDict(((i // 10, i % 10), torch.empty(n)) for i, n in enumerate(sizes))
    with cpu_reference():
        from tinytron.distributed.zero1.distributed_optimizer import partition_tensors as ref_fn

        ref, _ = ref_fn(td, ranks_map=ranks_map, num_parts=parts)
    ours, _ = partition_tensors(td, ranks_map=ranks_map, num_parts=parts)
    assert ours == ref
