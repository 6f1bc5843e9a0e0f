"""Memory-pruning K/V compaction (the gather side of adaptive context management).

The reference keeps only the retained history frames before its KV-cache
recompute: ``latents[:, :, selected_frame_indices]``
(hy-worldplay/patches/0001-integrate-acceleration.patch:3213-3221) and the
memory assembly from ``selected_index`` (matrix-game-3.0 patch :447-457). On
K/V that is a frame gather: ``dst[:, :, f] = pool[:, :, frame_ids[f]]`` for
frames of ``LH * LW`` tokens.

Two forms:

* :func:`gather_kv` — a coalesced 16-byte-vector copy into a contiguous
  compacted K/V buffer (``li_gather_frames``);
* the same frame list passed as ``frame_ids`` to ``kernels.pool_blocks`` /
  ``kernels.tile_pool``, which read the retained frames of the pool directly
  while pooling or tiling (no intermediate copy).
"""

from __future__ import annotations

from typing import Optional, Sequence, Union

import torch

from . import kernels as K


def _ids(frame_ids: Union[torch.Tensor, Sequence[int]], device) -> torch.Tensor:
    if isinstance(frame_ids, torch.Tensor):
        return frame_ids.to(device=device, dtype=torch.int32).contiguous()
    return torch.tensor(list(frame_ids), dtype=torch.int32, device=device)


def gather_kv(k_pool: torch.Tensor, v_pool: torch.Tensor, frame_ids, latent_hw,
              k_out: Optional[torch.Tensor] = None, v_out: Optional[torch.Tensor] = None):
    """Compact the retained frames of a ``[B, H, F*HW, D]`` K/V pool, in order."""
    LH, LW = latent_hw
    ids = _ids(frame_ids, k_pool.device)
    k = K.gather_frames(k_pool, ids, LH * LW, out=k_out)
    v = K.gather_frames(v_pool, ids, LH * LW, out=v_out)
    return k, v
