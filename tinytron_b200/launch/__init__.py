"""Command-line entry points (reference: scripts/debug/{pretrain,inference,rl}.py,
scripts/debug/pretrain.sh presets, scripts/autotune.sh).

    torchrun --nproc-per-node 8 -m tinytron_b200.launch.pretrain [training flags]
    python -m tinytron_b200.launch.pretrain --preset 1.3B --sep_size 1 ...
    torchrun --nproc-per-node 8 -m tinytron_b200.launch.inference --init_from_scratch --sep_size 8 ...
    torchrun --nproc-per-node 2 -m tinytron_b200.launch.rl --use_mock_data ...
    python -m tinytron_b200.launch.autotune --preset 0.25B --sep-sizes 1 2 --batch-sizes 4 8
    bash tinytron_b200/launch/pretrain.sh        (env-driven, same knobs as the reference launcher)
"""
