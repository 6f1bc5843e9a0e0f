"""Acceleration presets and the ``attn_param`` flag surface for HY-WorldPlay.

Mirrors ``WorldPlayAccelerationConfig`` (hy-worldplay/files/worldplay_acceleration_config.py:18-210):
the same preset names (off, context, sparse, cache, all), field names, defaults,
override guards and ``to_attn_param()`` keys, so the upstream pipeline can keep
passing ``pipe.transformer.attn_param.update(cfg.to_attn_param())``. The field
values are the reference's published defaults; the sparse-attention ones are
what the HY attention dispatch turns into ``sparse_params``
(``decode_params`` / ``prefill_params`` below).
"""

from __future__ import annotations

from dataclasses import dataclass, fields
from typing import Dict, Tuple

PRESETS = ("off", "context", "sparse", "cache", "all")

_SPARSE_OFF = dict(enable_sparse_attention=False, enable_prefill_sparse=False, enable_decode_sparse=False)
_TEMPORAL_CONTEXT = dict(context_mode="temporal", context_memory_frames=20, context_temporal_size=12,
                         enable_spatial_context_filter=False)

# Non-default fields of each preset (the defaults are the 'all' preset).
_PRESET_FIELDS: Dict[str, dict] = {
    "off": {**_SPARSE_OFF, **_TEMPORAL_CONTEXT, "enable_denoise_cache": False, "enable_timing": False},
    "context": {**_SPARSE_OFF, "enable_denoise_cache": False},
    "sparse": {**_TEMPORAL_CONTEXT, "enable_denoise_cache": False},
    "cache": {**_SPARSE_OFF, **_TEMPORAL_CONTEXT},
    "all": {},
}


@dataclass
class WorldPlayAccelerationConfig:
    preset: str = "all"
    # sparse attention
    enable_sparse_attention: bool = True
    enable_prefill_sparse: bool = True
    enable_decode_sparse: bool = True
    sparse_decode_start_chunk: int = 3
    sparse_prefill_topk_ratio: float = 0.3
    sparse_decode_topk_ratio: float = 0.175
    sparse_tile_size: Tuple[int, int, int] = (4, 8, 4)
    sparse_recent_protect: int = 4
    # adaptive context management
    context_mode: str = "spatial_temporal"
    context_memory_frames: int = 12
    context_temporal_size: int = 4
    enable_spatial_context_filter: bool = True
    spatial_similarity_threshold: float = 0.7
    context_pred_latent_size: int = 4
    # denoising cache
    enable_denoise_cache: bool = True
    denoise_cache_steps: Tuple[int, ...] = (1, 2)
    denoise_cache_similarity_threshold: float = 0.7
    # diagnostics
    enable_timing: bool = True
    enable_l1_diagnostics: bool = False

    @classmethod
    def from_preset(cls, preset: str) -> "WorldPlayAccelerationConfig":
        """Build the configuration of a named preset (``ValueError`` if unknown)."""
        name = (preset or "all").lower()
        if name not in _PRESET_FIELDS:
            raise ValueError(f"Unknown acceleration preset '{name}'. Choose from: {', '.join(PRESETS)}.")
        cfg = cls(preset=name)
        for key, value in _PRESET_FIELDS[name].items():
            setattr(cfg, key, value)
        return cfg

    def apply_overrides(self, **overrides) -> "WorldPlayAccelerationConfig":
        """Set the given non-``None`` fields, then re-apply the consistency guards:
        sparse attention off turns prefill/decode sparsity off; 'none'/'temporal'
        context turns the spatial filter off."""
        allowed = {"enable_sparse_attention", "enable_prefill_sparse", "enable_decode_sparse", "context_mode",
                   "context_memory_frames", "context_temporal_size", "enable_spatial_context_filter",
                   "spatial_similarity_threshold", "enable_denoise_cache", "enable_l1_diagnostics"}
        for key, value in overrides.items():
            if key not in allowed:
                raise TypeError(f"apply_overrides() got an unexpected keyword argument '{key}'")
            if value is not None:
                setattr(self, key, value)
        if not self.enable_sparse_attention:
            self.enable_prefill_sparse = False
            self.enable_decode_sparse = False
        if self.context_mode in ("none", "temporal"):
            self.enable_spatial_context_filter = False
        return self

    def to_attn_param(self) -> Dict[str, object]:
        """The fields the sparse-attention backend consumes (same keys as the reference)."""
        on = self.enable_sparse_attention
        return {
            "enable_sparse": on,
            "enable_prefill_sparse": on and self.enable_prefill_sparse,
            "enable_decode_sparse": on and self.enable_decode_sparse,
            "sparse_decode_start_chunk": self.sparse_decode_start_chunk,
            "sparse_prefill_topk_ratio": self.sparse_prefill_topk_ratio,
            "sparse_decode_topk_ratio": self.sparse_decode_topk_ratio,
            "sparse_tile_size": list(self.sparse_tile_size),
            "sparse_recent_protect": self.sparse_recent_protect,
            "enable_denoise_cache": self.enable_denoise_cache,
            "denoise_cache_steps": tuple(self.denoise_cache_steps),
            "enable_l1_diagnostics": self.enable_l1_diagnostics,
        }


def sparse_params_from_attn_param(attn_param: Dict[str, object]):
    """``(decode_params, prefill_params)`` exactly as the patched HY attention
    dispatch builds them (hy-worldplay/patches/0001-integrate-acceleration.patch:598-626)."""
    ap = attn_param or {}
    tile = tuple(ap.get("sparse_tile_size", (4, 8, 4)))
    prefill = {"tile_size": tile, "topk_ratio": ap.get("sparse_prefill_topk_ratio", 0.3),
               "sim_metric": "scaled_dot_product"}
    decode = {"tile_size": tile, "topk_ratio": ap.get("sparse_decode_topk_ratio", 0.175),
              "recent_protect": ap.get("sparse_recent_protect", 4), "sim_metric": "scaled_dot_product"}
    return decode, prefill


def config_fields():
    return [f.name for f in fields(WorldPlayAccelerationConfig)]
