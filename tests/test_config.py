"""The acceleration-preset flag surface (pure host logic)."""

import pytest

from light_interaction_project_b200.worldplay_acceleration_config import (
    PRESETS, WorldPlayAccelerationConfig, sparse_params_from_attn_param)


def test_defaults_are_the_all_preset():
    a = WorldPlayAccelerationConfig()
    b = WorldPlayAccelerationConfig.from_preset("all")
    assert a.to_attn_param() == b.to_attn_param()
    assert a.sparse_tile_size == (4, 8, 4) and a.sparse_decode_topk_ratio == 0.175
    assert a.sparse_prefill_topk_ratio == 0.3 and a.sparse_recent_protect == 4 and a.sparse_decode_start_chunk == 3


@pytest.mark.parametrize("name", PRESETS)
def test_presets(name):
    cfg = WorldPlayAccelerationConfig.from_preset(name.upper())
    ap = cfg.to_attn_param()
    sparse_on = name in ("sparse", "all")
    assert ap["enable_sparse"] is sparse_on
    assert ap["enable_prefill_sparse"] is sparse_on and ap["enable_decode_sparse"] is sparse_on
    assert ap["enable_denoise_cache"] is (name in ("cache", "all"))
    if name in ("off", "sparse", "cache"):
        assert cfg.context_mode == "temporal" and cfg.context_memory_frames == 20
    assert cfg.enable_timing is (name != "off")


def test_unknown_preset():
    with pytest.raises(ValueError, match="Unknown acceleration preset"):
        WorldPlayAccelerationConfig.from_preset("turbo")


def test_override_guards():
    cfg = WorldPlayAccelerationConfig().apply_overrides(enable_sparse_attention=False, context_mode="none")
    assert not cfg.enable_prefill_sparse and not cfg.enable_decode_sparse
    assert not cfg.enable_spatial_context_filter
    ap = cfg.to_attn_param()
    assert ap["enable_prefill_sparse"] is False
    with pytest.raises(TypeError):
        cfg.apply_overrides(sparse_tile_size=(1, 1, 1))


def test_attn_param_to_sparse_params():
    decode, prefill = sparse_params_from_attn_param(WorldPlayAccelerationConfig().to_attn_param())
    assert decode == {"tile_size": (4, 8, 4), "topk_ratio": 0.175, "recent_protect": 4,
                      "sim_metric": "scaled_dot_product"}
    assert prefill == {"tile_size": (4, 8, 4), "topk_ratio": 0.3, "sim_metric": "scaled_dot_product"}
