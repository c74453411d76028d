"""Optimizer options (CPU): element-wise gradient clipping, weight_decay_final checks."""

import pytest
import torch

from burn_dragon_b200.config import DragonConfig, training_config_from_dict
from burn_dragon_b200.models.bdh import BDH
from burn_dragon_b200.train.optim import FusedAdamW


def _model():
    return BDH(DragonConfig(n_layer=1, n_embd=16, n_head=2, mlp_internal_dim_multiplier=4, vocab_size=32,
                            dropout=0.0), seed=4)


def test_grad_clip_value_clamps_every_element():
    a, b = _model(), _model()
    g = 10 * torch.randn_like(a.store.grad)
    for m in (a, b):
        m.store.grad.copy_(g)
    FusedAdamW(a.store, lr=1e-2, grad_clip_value=0.5).step()
    b.store.grad.copy_(g.clamp(-0.5, 0.5))
    FusedAdamW(b.store, lr=1e-2).step()
    torch.testing.assert_close(a.store.data, b.store.data)
    # a norm, when set, takes precedence (the reference checks the norm first)
    assert FusedAdamW(a.store, grad_clip_norm=1.0, grad_clip_value=0.5).clip_value is None


def test_optimizer_key_validation():
    cfg = training_config_from_dict({"optimizer": {"weight_decay_final": 0.01, "grad_clip_value": 1.0}})
    assert cfg.optimizer.weight_decay_final == 0.01 and not cfg.extras
    with pytest.raises(ValueError):
        training_config_from_dict({"optimizer": {"weight_decay_final": -0.1}})
    with pytest.raises(ValueError):
        training_config_from_dict({"optimizer": {"grad_clip_value": 0.0}})


def test_predictive_coding_optimizer_name_is_retired():
    with pytest.raises(ValueError, match="retired"):
        training_config_from_dict({"optimizer": {"name": "predictive_coding"}})
    with pytest.raises(ValueError):
        training_config_from_dict({"optimizer": {"name": "lion"}})


def test_legacy_gdpo_flag_is_rejected():
    with pytest.raises(ValueError, match="training.gdpo.enabled"):
        training_config_from_dict({"training": {"gdpo": {"enabled": True}}})
    assert not training_config_from_dict({"training": {"gdpo": {"enabled": False}}}).extras


def test_tensor_parallel_partition_rules():
    base = {"model": {"n_head": 4, "n_embd": 32}, "parallel": {"mode": "tensor_parallel_neuron"}}

    def cfg(tensor):
        return training_config_from_dict({**base, "parallel": {**base["parallel"], "tensor": tensor}})

    cfg({"size": 2, "partition": "contiguous"})
    cfg({"size": 4, "partition": "head_aligned"})
    with pytest.raises(ValueError, match="head_aligned requires"):
        cfg({"size": 8, "partition": "head_aligned"})
    with pytest.raises(ValueError, match="must divide"):
        cfg({"size": 3})
    with pytest.raises(ValueError):
        cfg({"axis": "embedding"})


def test_eggroll_auto_population():
    from burn_dragon_b200.config import OptimizerConfig

    o = OptimizerConfig(name="eggroll", eggroll={"population": {"population_size": 64, "population_chunk_size": 16,
                                                                 "rank": 2}},
                        eggroll_auto_population={"enabled": True, "population_per_batch": 96})
    r = o.apply_auto_eggroll_population(6)  # 6 x 96 = 576 -> the next power of two, 1024
    assert r["resolved_population_size"] == 1024 and r["resolved_population_chunk_size"] == 16
    assert o.eggroll["population"]["population_size"] == 1024 and o.eggroll["population"]["rank"] == 2
    o = OptimizerConfig(name="eggroll", eggroll_auto_population={
        "enabled": True, "min_population_size": 8, "max_population_size": 256, "population_per_batch": 1024,
        "population_chunk_size": 32, "prefer_power_of_two": False})
    r = o.apply_auto_eggroll_population(8)
    assert (r["resolved_population_size"], r["resolved_population_chunk_size"]) == (256, 32)
    assert OptimizerConfig(eggroll_auto_population={"enabled": True}).apply_auto_eggroll_population(4) is None
