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


class KeyPoolCache:
    """Selection-ready pooled keys of a resident K buffer (extension, no reference
    counterpart: the reference re-pools all of K on every call,
    ``ar_sparse_operation.py:329-335``, ``bi_sparse_operation.py:289-296``).

    Within one query chunk's denoising steps the memory frames' K is constant and
    only the current chunk's frames change. :meth:`refresh` pools every key block
    on its first call and afterwards only the block rows from
    ``changed_from_frame`` on (rounded down to a block-row boundary). For
    ``cosine`` the stored rows are normalised in the same launch. The rows are the
    same bits a full re-pool gives, so selection is unchanged.
    """

    def __init__(self, latent_hw, tile, metric: str = "cosine"):
        self.latent_hw = tuple(latent_hw)
        self.tile = tuple(int(t) for t in tile)
        self.metric = metric
        self.pool: Optional[torch.Tensor] = None
        self._shape = None

    def pool_job(self, k_vis: torch.Tensor, changed_from_frame: int = 0):
        """The pooling work :meth:`refresh` would launch, as a
        ``kernels.pool_blocks_multi`` job (``None`` when nothing changed), so a
        caller can pool these rows together with other pools in one launch. The
        cache counts as refreshed once that job has run."""
        LH, LW = self.latent_hw
        HW = LH * LW
        if k_vis.shape[2] % HW:
            raise ValueError("k_vis length must be a whole number of latent frames")
        T = k_vis.shape[2] // HW
        shape = (k_vis.shape[0], k_vis.shape[1], T, k_vis.shape[3], k_vis.dtype, k_vis.device)
        if self.pool is None or shape != self._shape:
            nt, nh, nw = K.grid_blocks(T, LH, LW, self.tile)
            self.pool = torch.empty((k_vis.shape[0], k_vis.shape[1], nt * nh * nw, k_vis.shape[3]),
                                    device=k_vis.device, dtype=k_vis.dtype)
            self._shape = shape
            changed_from_frame = 0
        tt = self.tile[0]
        f0 = (max(0, min(int(changed_from_frame), T)) // tt) * tt
        if f0 >= T:
            return None
        _, nh, nw = K.grid_blocks(T, LH, LW, self.tile)
        return dict(src=k_vis[:, :, f0 * HW:], T=T - f0, LH=LH, LW=LW, tile=self.tile, out=self.pool,
                    block_offset=(f0 // tt) * nh * nw, normalized=self.metric == "cosine")

    def refresh(self, k_vis: torch.Tensor, changed_from_frame: int = 0) -> "KeyPoolCache":
        job = self.pool_job(k_vis, changed_from_frame)
        if job is not None:
            K.pool_blocks(job["src"], job["T"], job["LH"], job["LW"], job["tile"], normalized=job["normalized"],
                          out=job["out"], block_offset=job["block_offset"])
        return self

    def selection_pool(self, metric: str) -> torch.Tensor:
        """The key pool the selection reads for ``metric`` (normalised for cosine)."""
        if self.pool is None:
            raise RuntimeError("KeyPoolCache.refresh() has not been called")
        if metric != self.metric:
            raise ValueError(f"cache built for metric {self.metric!r}, selection uses {metric!r}")
        return self.pool
