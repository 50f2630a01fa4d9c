"""Sharding plans (parameter specs) and their resolution from job configs."""

import torch

from representax_b200.models.bert import BertConfig, BertEncoder
from representax_b200.parallel.sharding import (
    ShardingPlan,
    fsdp_partition_spec,
    parameter_specs_from_rules,
    plan_from_config,
)


def test_fsdp_partition_spec_rules():
    assert fsdp_partition_spec((768,), axis_name="data", axis_size=8) == ()
    assert fsdp_partition_spec((3072, 768), axis_name="data", axis_size=8, minimum_elements=1) == ("data", None)
    assert fsdp_partition_spec((30522, 768), axis_name="data", axis_size=8, minimum_elements=1) == (None, "data")
    assert fsdp_partition_spec((30522, 767), axis_name="data", axis_size=8, minimum_elements=1) == ()
    assert fsdp_partition_spec((64, 64), axis_name="data", axis_size=8, minimum_elements=2 ** 18) == ()
    assert fsdp_partition_spec((3072, 768), axis_name="data", axis_size=1) == ()


def test_rules_first_match_wins():
    shapes = {"layers.0.qkv_weight": (2304, 768), "layers.0.qkv_bias": (2304,), "pooler_weight": (768, 768)}
    specs = parameter_specs_from_rules(shapes, [(r"qkv_weight", ("data", None)), (r"layers", ())], ("data", None))
    assert specs == {"layers.0.qkv_weight": ("data", None), "layers.0.qkv_bias": (), "pooler_weight": ("data", None)}


def test_plans_from_configs():
    from representax_b200.config import CustomShardingConfig, DDPConfig, FSDPConfig, PartitionRuleConfig

    model = BertEncoder(BertConfig(vocab_size=1024, hidden_size=128, num_hidden_layers=1, num_attention_heads=2,
                                   intermediate_size=512, max_position_embeddings=64))
    assert plan_from_config(DDPConfig(), model, 8).kind == "ddp"
    assert not plan_from_config(DDPConfig(), model, 8).sharded_optimizer
    fsdp = plan_from_config(FSDPConfig(minimum_parameter_elements=2 ** 15), model, 8)
    assert fsdp.sharded_optimizer and fsdp.has_sharded_parameters
    assert fsdp.parameter_specs["embeddings.word"] == ("data", None)
    assert 0 < fsdp.sharded_fraction(model) <= 1
    custom = plan_from_config(CustomShardingConfig(parameter_axes=("data",), parameter_rules=(
        PartitionRuleConfig(pattern="ffn_in_weight", axes=("data", None)),)), model, 8)
    assert custom.parameter_specs["layers.0.ffn_in_weight"] == ("data", None)
    assert custom.parameter_specs["layers.0.qkv_weight"] == ()
    assert ShardingPlan.zero(1).sharded_optimizer is False
