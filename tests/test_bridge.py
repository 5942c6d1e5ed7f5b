"""Bridge layout / planner / materializer / checkpoint-reshard tests (semantics of the
reference's tests/test_bridge_layout.py, written against this package)."""
import tempfile
from dataclasses import replace
from pathlib import Path
from unittest import mock

import pytest
import torch

from tinytron_b200.bridge import (BridgeContext, LayoutIndex, LayoutPlanner, ParallelSpec, Placement, RankCoord,
                                  RoutedMaterializer, ShardSpec, StateDictTensorStore, build_tinytron_canonical_layout,
                                  build_tinytron_inference_layout, build_tinytron_training_layout)
from tinytron_b200.bridge.layout import intersect_slices, local_slices
from tinytron_b200.models.config import ModelConfig


def moe_cfg():
    return ModelConfig(block_size=16, vocab_size=32, num_layer=1, num_attention_heads=4, num_key_value_heads=2,
                       hidden_size=8, intermediate_size=16, use_moe=True, num_experts=4, num_experts_per_tok=2,
                       moe_intermediate_size=4)


def test_experts_sharded_by_sep_rank():
    lay = build_tinytron_training_layout(moe_cfg(), ParallelSpec(1, 2, "training"))
    sh = lay.shards_for("blocks.0.mlp.experts_gate_weights")
    assert [s.global_slices[0] for s in sh] == [(0, 2), (2, 4)]
    assert [s.local_shape for s in sh] == [(2, 4, 8), (2, 4, 8)]
    assert {s.axis_tags for s in sh} == {("expert",)}


def test_training_to_inference_plan_across_sep_change():
    cfg = moe_cfg()
    plan = LayoutPlanner().plan(build_tinytron_training_layout(cfg, ParallelSpec(2, 4, "training")),
                                build_tinytron_inference_layout(cfg, ParallelSpec(1, 2, "inference"), shard_qkv=True))
    ex = [m for m in plan if m.param_name == "blocks.0.mlp.experts_gate_weights"]
    q = [m for m in plan if m.param_name == "blocks.0.attn.q_proj.weight"]
    assert [m.global_slices[0] for m in ex] == [(0, 1), (1, 2), (2, 3), (3, 4)]
    assert [m.src.rank for m in ex] == [0, 1, 2, 3]
    assert [m.dst.rank for m in ex] == [0, 0, 1, 1]
    assert [m.global_slices[0] for m in q] == [(0, 4), (4, 8)]
    assert [m.dst.rank for m in q] == [0, 1]


def test_same_rank_source_preferred():
    cfg = replace(moe_cfg(), inference_shard_qkv=True)
    plan = LayoutPlanner().plan(build_tinytron_training_layout(cfg, ParallelSpec(1, 2, "training")),
                                build_tinytron_inference_layout(cfg, ParallelSpec(1, 2, "inference"), shard_qkv=True))
    q = [m for m in plan if m.param_name == "blocks.0.attn.q_proj.weight"]
    assert [m.src.rank for m in q] == [0, 1] and [m.dst.rank for m in q] == [0, 1]


def test_balanced_planner_spreads_replicated_sources():
    """With balancing, the DP replicas of the expert shards share the sending, every
    target region is still covered exactly once, and local copies stay preferred."""
    from tinytron_b200.bridge.planner import group_by_rank_pair

    cfg = moe_cfg()
    src = build_tinytron_training_layout(cfg, ParallelSpec(2, 4, "training"))
    dst = build_tinytron_inference_layout(cfg, ParallelSpec(1, 2, "inference"), shard_qkv=True)
    plain, bal = LayoutPlanner().plan(src, dst), LayoutPlanner(balance_sources=True).plan(src, dst)
    key = lambda m: (m.param_name, m.dst.rank, m.global_slices)  # noqa: E731
    assert sorted(map(key, plain)) == sorted(map(key, bal))  # same pieces, possibly other sources

    def busiest(plan):
        sent = {}
        for m in plan:
            if m.src.rank != m.dst.rank:
                sent[m.src.rank] = sent.get(m.src.rank, 0) + m.numel
        return max(sent.values())

    assert busiest(bal) < busiest(plain)
    assert all(m.src.rank == m.dst.rank for m in bal if m.param_name == "blocks.0.attn.q_proj.weight")
    pairs = group_by_rank_pair(bal)
    assert sum(len(v) for v in pairs.values()) == len(bal)
    assert list(pairs) == sorted(pairs)


def test_canonical_to_inference_slices_qkv():
    cfg = moe_cfg()
    plan = LayoutPlanner().plan(build_tinytron_canonical_layout(cfg),
                                build_tinytron_inference_layout(cfg, ParallelSpec(1, 2, "inference"), shard_qkv=True))
    for name, want in [("q_proj", [(0, 4), (4, 8)]), ("k_proj", [(0, 2), (2, 4)]), ("v_proj", [(0, 2), (2, 4)])]:
        assert [m.global_slices[0] for m in plan if m.param_name == f"blocks.0.attn.{name}.weight"] == want


def test_uncovered_target_rejected():
    sp = Placement("src", 0, RankCoord.from_axes(replica=0))
    dp = Placement("dst", 0, RankCoord.from_axes(replica=0))
    src = LayoutIndex.from_shards("s", [ShardSpec("w", (4, 2), ((0, 2), (0, 2)), sp)])
    dst = LayoutIndex.from_shards("d", [ShardSpec("w", (4, 2), ((0, 4), (0, 2)), dp)])
    with pytest.raises(ValueError, match="does not cover target shard"):
        LayoutPlanner().plan(src, dst)


def test_slice_helpers():
    ov = intersect_slices(((0, 4), (0, 8)), ((2, 6), (3, 5)))
    assert ov == ((2, 4), (3, 5))
    assert local_slices(((0, 4), (0, 8)), ov) == ((2, 4), (3, 5))
    assert local_slices(((2, 6), (3, 5)), ov) == ((0, 2), (0, 2))


def test_materializer_copies_overlapping_slices():
    sp = Placement("src", 0, RankCoord.from_axes(replica=0))
    d0 = Placement("dst", 0, RankCoord.from_axes(replica=0))
    d1 = Placement("dst", 1, RankCoord.from_axes(replica=1))
    full = torch.arange(24.0).view(6, 4)
    src = LayoutIndex.from_shards("s", [ShardSpec("w", (6, 4), ((0, 6), (0, 4)), sp)])
    dst = LayoutIndex.from_shards("d", [ShardSpec("w", (6, 4), ((0, 3), (0, 4)), d0),
                                        ShardSpec("w", (6, 4), ((3, 6), (0, 4)), d1)])
    out = StateDictTensorStore()
    RoutedMaterializer().materialize(LayoutPlanner().plan(src, dst),
                                     BridgeContext(StateDictTensorStore({sp: {"w": full}}), out))
    assert torch.equal(out.state_dict_for(d0)["w"], full[:3])
    assert torch.equal(out.state_dict_for(d1)["w"], full[3:])


def _filled(layout, placement, rank):
    sd = {}
    for s in layout.local_shards(placement):
        n = 1
        for d in s.local_shape:
            n *= d
        sd[s.param_name] = (torch.arange(n, dtype=torch.float32) + rank * 1000).view(s.local_shape)
    return sd


def test_reshard_sep4_files_to_sep2_training_and_inference():
    from tinytron_b200.inference import checkpoint as icp
    from tinytron_b200.training import checkpoint as tcp

    cfg = moe_cfg()
    src_spec = ParallelSpec(1, 4, "training")
    src = build_tinytron_training_layout(cfg, src_spec)
    with tempfile.TemporaryDirectory() as td:
        prefix = str(Path(td) / "00010")
        for p in src.placements():
            torch.save(_filled(src, p, p.rank), tcp.checkpoint_model_shard_path(prefix, p.rank))
        torch.save(_filled(src, src.placements()[0], 0), f"{prefix}_model.pt")
        meta = {"model_sharded": True, "model_layout": {"layout_kind": "training", "parallel": src_spec.__dict__}}
        torch.save(meta, f"{prefix}_meta.pt")
        for rank in (0, 1):
            cur = ParallelSpec(1, 2, "training")
            pl = [p for p in build_tinytron_training_layout(cfg, cur).placements() if p.rank == rank][0]
            with mock.patch.object(tcp, "current_tinytron_parallel_spec", return_value=cur), \
                    mock.patch.object(tcp, "current_tinytron_placement", return_value=pl):
                sd = tcp.load_model_state_dict_for_training(prefix, cfg, rank, meta)
            g = sd["blocks.0.mlp.experts_gate_weights"]
            assert g.shape == (2, 4, 8)
            # experts 2r, 2r+1 came from source ranks 2r, 2r+1 (value offset rank*1000)
            assert g[0].flatten()[0].item() == 2 * rank * 1000 and g[1].flatten()[0].item() == (2 * rank + 1) * 1000
        icfg = replace(cfg, inference_shard_qkv=True)
        cur = ParallelSpec(1, 2, "inference")
        pl = [p for p in build_tinytron_inference_layout(icfg, cur, True).placements() if p.rank == 1][0]
        with mock.patch.object(icp, "current_tinytron_parallel_spec", return_value=cur), \
                mock.patch.object(icp, "current_tinytron_placement", return_value=pl):
            sd = icp.load_model_state_dict_for_inference(f"{prefix}_model.pt", icfg)
        assert sd["blocks.0.attn.q_proj.weight"].shape == (4, 8)
        # q is replicated in training: destination rank 1 reads rank 1's own copy (same-rank preference)
        full_q = _filled(src, src.placements()[1], 1)["blocks.0.attn.q_proj.weight"]
        assert torch.equal(sd["blocks.0.attn.q_proj.weight"], full_q[4:])


def test_corrupt_shard_detected():
    from tinytron_b200.training import checkpoint as tcp

    with tempfile.TemporaryDirectory() as td:
        path = str(Path(td) / "00001_model_rank00000.pt")
        model = torch.nn.Linear(4, 4)
        torch.save(model.state_dict(), path)
        tcp._write_crc(path)
        with open(path, "r+b") as f:
            f.seek(-8, 2)
            f.write(b"\x00\x01\x02\x03\x04\x05\x06\x07")
        with pytest.raises(tcp.CheckpointCorruptError):
            tcp.verify_checksum(path)


def _reshard_with(api, cfg, files_prefix, src_spec, dst_layout, rank):
    """Materialize placement `rank` of dst_layout from the source shard files with one
    framework's bridge API (`api` is this package's or the reference's bridge module)."""
    src = api.build_tinytron_training_layout(cfg, src_spec)
    pl = [p for p in dst_layout.placements() if p.rank == rank][0]
    store = api.StateDictShardFileStore(lambda p: f"{files_prefix}_model_rank{int(p.rank or 0):05d}.pt")
    out = api.StateDictTensorStore()
    api.RoutedMaterializer().materialize(api.LayoutPlanner().plan(src, api.localize_layout(dst_layout, pl)),
                                         api.BridgeContext(src_store=store, dst_store=out))
    return out.state_dict_for(pl), dst_layout.local_shards(pl)


def test_reshard_matches_reference_bridge_and_ground_truth():
    """SEP=4 training shards cut from one full state dict, resharded to SEP=2 training,
    SEP=2 q/k/v-sharded inference and SEP=1 inference by this package's bridge and by the
    reference's: every destination shard equals its slice of the full tensors in both."""
    import ref_oracle
    from tinytron_b200 import bridge as ours
    from tinytron_b200.bridge.layout import to_torch_slices

    if not ref_oracle.available():
        pytest.skip("reference not installed under baseline/_ref")
    cfg = moe_cfg()
    g = torch.Generator().manual_seed(0)
    full = {}
    for s in ours.build_tinytron_canonical_layout(cfg).local_shards(
            ours.build_tinytron_canonical_layout(cfg).placements()[0]):
        full[s.param_name] = torch.randn(s.global_shape, generator=g)
    src_spec = ParallelSpec(1, 4, "training")
    src = build_tinytron_training_layout(cfg, src_spec)
    with tempfile.TemporaryDirectory() as td, ref_oracle.cpu_reference():
        from tinytron import bridge as ref
        from tinytron.model.config import ModelConfig as RefCfg

        rcfg = RefCfg(**{k: v for k, v in cfg.__dict__.items() if k in RefCfg.__dataclass_fields__})
        prefix = str(Path(td) / "00004")
        for p in src.placements():  # real replicas: every rank's copy of a replicated tensor is equal
            torch.save({s.param_name: full[s.param_name][to_torch_slices(s.global_slices)].clone()
                        for s in src.local_shards(p)}, f"{prefix}_model_rank{p.rank:05d}.pt")
        targets = [
            ("train sep2", lambda api, c: api.build_tinytron_training_layout(c, api.ParallelSpec(1, 2, "training")),
             (0, 1)),
            ("infer sep2 qkv", lambda api, c: api.build_tinytron_inference_layout(
                c, api.ParallelSpec(1, 2, "inference"), True), (0, 1)),
            ("infer sep1", lambda api, c: api.build_tinytron_inference_layout(
                c, api.ParallelSpec(1, 1, "inference"), False), (0,)),
        ]
        for name, make, ranks in targets:
            for rank in ranks:
                o_sd, o_shards = _reshard_with(ours, cfg, prefix, src_spec, make(ours, cfg), rank)
                r_sd, _ = _reshard_with(ref, rcfg, prefix, ref.ParallelSpec(1, 4, "training"), make(ref, rcfg), rank)
                assert set(o_sd) == set(r_sd), (name, rank)
                names = [s.param_name for s in o_shards]
                assert any("experts" in n for n in names) and any(".attn." in n for n in names), (name, names)
                for s in o_shards:
                    want = full[s.param_name][to_torch_slices(s.global_slices)]
                    assert torch.equal(o_sd[s.param_name], want), (name, rank, s.param_name)
                    assert torch.equal(r_sd[s.param_name], want), (name, rank, s.param_name, "reference")
