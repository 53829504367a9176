"""MLX quantized safetensors checkpoints: format round trip, the loader's errors, the
quantization entry, and a checkpoint of the verify stack sharded for tensor parallelism
(the same shards as the synthetic weights), loaded on the GPU to the same forward."""
from __future__ import annotations

import json
from dataclasses import replace

import pytest
import torch

import mlx_checkpoint as mc
import verify_stack as vs


def test_safetensors_round_trip(tmp_path):
    g = torch.Generator().manual_seed(0)
    t = {"a.bf16": torch.randn(3, 5, generator=g).to(torch.bfloat16),
         "b.f32": torch.randn(7, generator=g),
         "c.words": torch.randint(-2 ** 31, 2 ** 31 - 1, (4, 6), dtype=torch.int32, generator=g),
         "d.i32": torch.arange(10, dtype=torch.int32)}
    mc.save_file(tmp_path / "x.safetensors", t, metadata={"format": "mlx"}, u32_names={"c.words"})
    header, start = mc.read_header(tmp_path / "x.safetensors")
    assert header["c.words"]["dtype"] == "U32" and header["a.bf16"]["dtype"] == "BF16" and start % 8 == 0
    back = mc.load_file(tmp_path / "x.safetensors")
    for k, v in t.items():
        assert back[k].dtype == v.dtype and torch.equal(back[k], v), k


def test_loader_errors(tmp_path):
    with pytest.raises(mc.CheckpointError, match="No config.json"):
        mc.load_directory(tmp_path)
    (tmp_path / "config.json").write_text("{}")
    with pytest.raises(mc.CheckpointError, match="No .safetensors"):
        mc.load_directory(tmp_path)
    bad = tmp_path / "model.safetensors"
    bad.write_bytes(b"\x05\x00")
    with pytest.raises(mc.CheckpointError, match="truncated"):
        mc.load_directory(tmp_path)


def test_quantization_entry_and_shape_check():
    cfg = {"quantization": {"group_size": 64, "bits": 4, "model.layers.0.mlp.down_proj": {"group_size": 32, "bits": 8}}}
    assert mc.quantization_of(cfg, "model.layers.1.mlp.down_proj") == (64, 4)
    assert mc.quantization_of(cfg, "model.layers.0.mlp.down_proj") == (32, 8)
    q = vs.random_quant(torch.Generator().manual_seed(1), 16, 256, 64, 4, "cpu")
    t = {"p.weight": q.w, "p.scales": q.scales, "p.biases": q.biases}
    assert mc.quantized_layer(t, {"quantization": {"group_size": 64, "bits": 4}}, "p").K == 256
    with pytest.raises(mc.CheckpointError):
        mc.quantized_layer(t, {"quantization": {"group_size": 64, "bits": 8}}, "p")
    with pytest.raises(mc.CheckpointError, match="missing"):
        mc.quantized_layer({"p.weight": q.w}, {"quantization": {"group_size": 64, "bits": 4}}, "p")


def _same_weights(a, b):
    assert len(a["layers"]) == len(b["layers"])
    for La, Lb in zip(a["layers"], b["layers"]):
        assert La.keys() == Lb.keys()
        for k in La:
            x, y = La[k], Lb[k]
            if isinstance(x, vs.Quant):
                assert (x.group, x.bits) == (y.group, y.bits)
                for f in ("w", "scales", "biases"):
                    assert torch.equal(getattr(x, f), getattr(y, f)), (k, f)
            elif isinstance(x, torch.Tensor):
                assert torch.equal(x, y), k
            else:
                assert x == y
    assert torch.equal(a["final_norm"], b["final_norm"])
    for f in ("w", "scales", "biases"):
        assert torch.equal(getattr(a["lm_head"], f), getattr(b["lm_head"], f))


@pytest.mark.parametrize("world", [1, 2])
def test_stack_checkpoint_shards_like_synthetic_weights(tmp_path, world):
    cfg = vs.TINY
    full = vs.build_rank_weights(cfg, vs.shard_plan(cfg, 0, 1), 0, "cpu")
    mc.save_stack_checkpoint(tmp_path, cfg, full, shard_bytes=1 << 20)
    assert len(list(tmp_path.glob("*.safetensors"))) > 1
    config, tensors = mc.load_directory(tmp_path)
    assert json.loads((tmp_path / "config.json").read_text())["quantization"] == {"group_size": 64, "bits": 4}
    for r in range(world):
        plan = vs.shard_plan(cfg, r, world)
        _same_weights(mc.stack_from_checkpoint(cfg, plan, config, tensors, "cpu"),
                      vs.build_rank_weights(cfg, plan, 0, "cpu"))


def test_stack_config_from_config_json(tmp_path):
    """The stack configuration comes back from a saved checkpoint's config.json, and the
    Qwen3.5 keys map onto config 4's stack; what the stack cannot take is rejected."""
    mc.save_stack_checkpoint(tmp_path, vs.TINY, vs.build_rank_weights(vs.TINY, vs.shard_plan(vs.TINY, 0, 1), 0,
                                                                        "cpu"))
    config, _ = mc.load_directory(tmp_path)
    assert mc.stack_config_from_json(config, context=vs.TINY.context, block=vs.TINY.block) == vs.TINY
    c4 = {"model_type": "qwen3_5", "hidden_size": 5120, "num_hidden_layers": 64, "intermediate_size": 17408,
          "full_attention_interval": 4, "linear_num_value_heads": 32, "linear_num_key_heads": 32,
          "linear_key_head_dim": 128, "linear_value_head_dim": 128, "linear_conv_kernel_dim": 4,
          "num_attention_heads": 24, "num_key_value_heads": 4, "head_dim": 256, "rms_norm_eps": 1e-6,
          "vocab_size": 248320, "rope_parameters": {"rope_type": "default", "rope_theta": 1.0e7,
                                                    "partial_rotary_factor": 0.25},
          "quantization": {"group_size": 64, "bits": 4}}
    assert mc.stack_config_from_json(c4, context=1024) == vs.CONFIG4
    # the reference's tiny fixture (TinyHybridTarget.swift:20-44): 2 key heads for 4 value
    # heads, and a 4-wide rotary span
    tiny = {**c4, "hidden_size": 64, "num_hidden_layers": 4, "intermediate_size": 128, "num_attention_heads": 4,
            "num_key_value_heads": 2, "head_dim": 16, "linear_num_value_heads": 4, "linear_num_key_heads": 2,
            "linear_key_head_dim": 32, "linear_value_head_dim": 32, "vocab_size": 64, "full_attention_interval": 2}
    with pytest.raises(mc.CheckpointError, match="rotary"):
        mc.stack_config_from_json(tiny, context=8)
    grouped = mc.stack_config_from_json({**tiny, "head_dim": 256}, context=8)  # rotary 0.25 x 256 = 64
    assert (grouped.gdn_heads, grouped.gdn_key_heads, grouped.gdn_kheads) == (4, 2, 2)
    with pytest.raises(mc.CheckpointError, match="key heads"):
        mc.stack_config_from_json({**tiny, "head_dim": 256, "linear_num_key_heads": 3}, context=8)
    with pytest.raises(mc.CheckpointError, match="hidden_size"):
        mc.stack_config_from_json({k: v for k, v in c4.items() if k != "hidden_size"}, context=8)


def test_fused_projection_given_as_parts(tmp_path):
    """A checkpoint that stores gate_proj and up_proj separately loads to the same
    [gate | up] shards as one storing the fused gate_up_proj."""
    cfg = vs.TINY
    full = vs.build_rank_weights(cfg, vs.shard_plan(cfg, 0, 1), 0, "cpu")
    mc.save_stack_checkpoint(tmp_path, cfg, full)
    config, tensors = mc.load_directory(tmp_path)
    I = cfg.intermediate
    for i in range(cfg.layers):
        pre = f"model.layers.{i}.mlp"
        for part, rows in (("gate_proj", slice(0, I)), ("up_proj", slice(I, 2 * I))):
            for f in ("weight", "scales", "biases"):
                tensors[f"{pre}.{part}.{f}"] = tensors[f"{pre}.gate_up_proj.{f}"][rows]
        for f in ("weight", "scales", "biases"):
            del tensors[f"{pre}.gate_up_proj.{f}"]
    plan = vs.shard_plan(cfg, 1, 2)
    _same_weights(mc.stack_from_checkpoint(cfg, plan, config, tensors, "cpu"), vs.build_rank_weights(cfg, plan, 0, "cpu"))


@pytest.mark.gpu
def test_stack_from_checkpoint_runs_the_same_forward(tmp_path, cuda):
    cfg = vs.TINY
    plan = vs.shard_plan(cfg, 0, 1)
    mc.save_stack_checkpoint(tmp_path, cfg, vs.build_rank_weights(cfg, plan, 0, cuda))
    config, tensors = mc.load_directory(tmp_path)
    w = mc.stack_from_checkpoint(cfg, plan, config, tensors, cuda)
    a = vs.VerifyStack(cfg, 0, 1, seed=0, device=cuda)
    b = vs.VerifyStack(cfg, 0, 1, seed=0, device=cuda, weights=w)
    hidden = vs.make_block(cfg, 0, cuda)
    assert torch.equal(a.forward(hidden), b.forward(hidden))
