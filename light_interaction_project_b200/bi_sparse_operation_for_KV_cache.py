"""Drop-in for HY-WorldPlay's ``bi_sparse_operation_for_KV_cache`` (bidirectional
prefill / KV-cache recompute path).

Reference: hy-worldplay/files/hyvideo/models/transformers/modules/bi_sparse_operation_for_KV_cache.py.
"""

from __future__ import annotations

import types

import torch

from . import _lib as L
from . import kernels as K
from .ar_sparse_operation import launch_kv_prep, launch_q_prep, launch_untile  # noqa: F401  (same surface)
from .pipeline import dense_attention, sparse_forward

HAS_TRITON = False
HAS_NATIVE = True

_DEFAULT_TILE = (4, 8, 4)  # bi_sparse_operation_for_KV_cache.py:347
_fallback_state = types.SimpleNamespace(current_chunk_index=0)


def get_infer_state():
    """The upstream inference state (``hyvideo.commons.infer_state``) when HY is
    importable, else a local stand-in whose ``current_chunk_index`` callers set."""
    try:
        from hyvideo.commons.infer_state import get_infer_state as upstream  # type: ignore
    except Exception:
        return _fallback_state
    return upstream()


def _pools(x, params):
    """4-D pooled input as is; 5-D tiled input ``[B,H,N,bs,D]`` pooled with the
    block-mean kernel (``:239-250`` take ``mean(dim=-2)``)."""
    if x.dim() == 5:
        B, H, N, bs, D = x.shape
        flat = x.reshape(B, H, N * bs, D)
        return K.pool_blocks(flat, N, 1, bs, (1, 1, bs)), bs
    tt, th, tw = params["tile_size"]
    return x, tt * th * tw


def generate_prefill_indices(q_in, k_in, text_len, grid_thw, params, device, q_block_offset=None):
    """Bidirectional block selection — ``bi_sparse_operation_for_KV_cache.py:220-296``.

    Protects every key block within 3D Manhattan distance 1 of the query block
    and keeps ``min(max(int(N_k * topk_ratio), 7), N_k)`` blocks. Like the
    reference it needs ``N_q == N_k``; ``q_block_offset`` (an extension) selects
    for a contiguous run of query rows placed at that key-grid position.
    """
    q_pool, bs = _pools(q_in, params)
    k_pool, _ = _pools(k_in, params)
    nq, nk = q_pool.shape[2], k_pool.shape[2]
    if q_block_offset is None and nq != nk:
        raise RuntimeError(f"bidirectional block selection needs N_q == N_k (got {nq} and {nk})")
    tile = (1, 1, bs) if q_in.dim() == 5 else params["tile_size"]
    p = K.select_params(L.SELECT_BIDIR, params.get("sim_metric", "cosine"), tile, grid_thw, grid_thw, text_len,
                        topk_ratio=params["topk_ratio"], min_budget=7, q_block_offset=q_block_offset or 0)
    return K.select_blocks(q_pool, k_pool, p)


def run_sparse_prefill_attention(q, k_txt, v_txt, k_vis, v_vis, block_idx, latent_hw, sparse_params):
    """One bidirectional (prefill) sparse-attention forward —
    ``bi_sparse_operation_for_KV_cache.py:301-395``. Dense for the first three
    chunks (``current_chunk_index < 3``) and for untileable query lengths.
    Device-side errors (a bounded wait that gave up; a block id out of range)
    do not raise here: the kernels record them in the device error word, which
    ``kernels.raise_device_errors()`` reads (and synchronises) at a step boundary.
    """
    current = getattr(get_infer_state(), "current_chunk_index", 0)
    LH, LW = latent_hw
    if current < 3 or q.shape[2] % (LH * LW) != 0:
        return dense_attention(q, torch.cat([k_txt, k_vis], dim=2), torch.cat([v_txt, v_vis], dim=2))
    return sparse_forward(q, k_txt, v_txt, k_vis, v_vis, latent_hw, sparse_params, L.SELECT_BIDIR, _DEFAULT_TILE,
                          ratio=sparse_params["topk_ratio"])
