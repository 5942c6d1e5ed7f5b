"""CLI compatibility with the reference: every option of the reference's training and
inference parsers exists here with the same default, type and choices, so a reference
command line runs unchanged.  Options added here (B200 extensions) are allowed.
Skipped when the reference is not installed under baseline/_ref."""
import argparse

import pytest

from ref_oracle import available, cpu_reference

pytestmark = pytest.mark.skipif(not available(), reason="reference not installed under baseline/_ref")


def _options(parser: argparse.ArgumentParser) -> dict:
    out = {}
    for a in parser._actions:
        if isinstance(a, argparse._HelpAction):
            continue
        for s in a.option_strings:
            out[s] = a
    return out


def _kind(a) -> str:
    return type(a).__name__


@pytest.mark.parametrize("which", ["training", "inference"])
def test_reference_options_exist_with_same_defaults(which):
    import importlib

    with cpu_reference():
        ref = importlib.import_module(f"tinytron.{which}.arguments").build_parser()
    ours = importlib.import_module(f"tinytron_b200.{which}.arguments").build_parser()
    ref_opts, our_opts = _options(ref), _options(ours)
    missing = sorted(set(ref_opts) - set(our_opts))
    assert not missing, f"reference options missing here: {missing}"
    for s, ra in ref_opts.items():
        oa = our_opts[s]
        assert _kind(oa) == _kind(ra), (s, _kind(oa), _kind(ra))
        assert oa.default == ra.default, (s, oa.default, ra.default)
        assert oa.type == ra.type, (s, oa.type, ra.type)
        if ra.choices is not None:
            assert oa.choices is not None and set(ra.choices) <= set(oa.choices), (s, oa.choices, ra.choices)


def test_reference_command_line_parses_the_same():
    """The reference launcher's flag set for the dense 1.3B preset parses to the same
    values in both parsers."""
    argv = ["--num_layer", "24", "--hidden_size", "2048", "--num_attention_heads", "16", "--num_key_value_heads",
            "4", "--intermediate_size", "5504", "--batch_size", "4", "--seq_len", "4096", "--total_batch_size",
            "65536", "--sep_size", "1", "--use_distributed_optimizer", "--use_mock_data", "--deterministic",
            "--init_std", "0.02"]
    with cpu_reference():
        from tinytron.training.arguments import parse_args as ref_parse

        ref = vars(ref_parse(argv))
    from tinytron_b200.training.arguments import parse_args

    ours = vars(parse_args(argv))
    for k, v in ref.items():
        assert k in ours and ours[k] == v, (k, ours.get(k), v)


def test_config_dataclasses_keep_the_reference_fields():
    """Every field of the reference's frozen config dataclasses exists here, and
    build_config of a reference command line gives the same values for them."""
    import dataclasses

    argv = ["--num_layer", "2", "--hidden_size", "64", "--num_attention_heads", "4", "--num_key_value_heads", "2",
            "--intermediate_size", "96", "--batch_size", "2", "--seq_len", "32", "--block_size", "32",
            "--vocab_size", "128", "--total_batch_size", "128", "--use_mock_data", "--max_steps", "3",
            "--warmup_steps", "1"]
    with cpu_reference():
        from tinytron.training import config as ref_cfg
        from tinytron.training.arguments import parse_args as ref_parse

        ref = ref_cfg.build_config(ref_parse(argv))
    from tinytron_b200.training import config as our_cfg
    from tinytron_b200.training.arguments import parse_args

    ours = our_cfg.build_config(parse_args(argv))
    for name in ("Config", "TrainingConfig", "LoggingConfig", "SeedConfig", "DataConfig", "OptimConfig",
                 "CheckpointConfig", "ParallelConfig"):
        ref_fields = {f.name for f in dataclasses.fields(getattr(ref_cfg, name))}
        our_fields = {f.name for f in dataclasses.fields(getattr(our_cfg, name))}
        assert ref_fields <= our_fields, (name, sorted(ref_fields - our_fields))

    def compare(r, o, path):
        for f in dataclasses.fields(r):
            rv, ov = getattr(r, f.name), getattr(o, f.name)
            if dataclasses.is_dataclass(rv):
                compare(rv, ov, f"{path}.{f.name}")
            else:
                assert ov == rv, (f"{path}.{f.name}", ov, rv)

    compare(ref, ours, "config")


@pytest.mark.parametrize("argv", [[], ["--use_moe", "--num_experts", "8", "--num_experts_per_tok", "2",
                                       "--moe_intermediate_size", "64", "--hidden_size", "128", "--num_layer", "3"]])
def test_model_config_builder_matches_reference(argv):
    """add_model_config_args / build_model_config give the same ModelConfig fields (and the
    reference's default config) for the same command line and overrides."""
    import dataclasses

    with cpu_reference():
        from tinytron.model import add_model_config_args as ref_add
        from tinytron.model import build_model_config as ref_build

        p = argparse.ArgumentParser()
        ref_add(p)
        ref = ref_build(p.parse_args(argv), block_size=256)
    from tinytron_b200.models import add_model_config_args, build_model_config

    p = argparse.ArgumentParser()
    add_model_config_args(p)
    ours = build_model_config(p.parse_args(argv), block_size=256)
    for f in dataclasses.fields(ref):
        assert getattr(ours, f.name) == getattr(ref, f.name), (f.name, getattr(ours, f.name), getattr(ref, f.name))
