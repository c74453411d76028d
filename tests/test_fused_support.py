"""Which model options the fused kernels implement (CPU): the trainer takes the
PyTorch path on CUDA for the rest instead of failing."""

from burn_dragon_b200.config import DragonConfig
from burn_dragon_b200.models.bdh_fused import fused_unsupported


def test_fused_support_matrix():
    base = dict(n_layer=1, n_embd=64, n_head=2, mlp_internal_dim_multiplier=4, vocab_size=64)
    assert fused_unsupported(DragonConfig(**base, dropout=0.0)) is None
    assert fused_unsupported(DragonConfig(**base, dropout=0.1)) == "dropout > 0"
    for kind in ("rms_norm", "dynamic_tanh", "derf"):
        assert fused_unsupported(DragonConfig(**base, dropout=0.0, norm_kind=kind)) is None
    assert fused_unsupported(DragonConfig(**base, dropout=0.0, rotary_embedding="pope")) == "PoPE"
    assert fused_unsupported(DragonConfig(**base, dropout=0.0, tie_input_output_embeddings=True)) == "a tied lm_head"


def test_data_transport_key_is_validated():
    from burn_dragon_b200.config import training_config_from_dict

    cfg = training_config_from_dict({"parallel": {"mode": "ddp", "data": {"transport": "nvls"}}})
    cfg.validate()
    import pytest

    with pytest.raises(ValueError, match="transport"):
        training_config_from_dict({"parallel": {"mode": "ddp", "data": {"transport": "ib"}}}).validate()
