"""The sparse-attention pipeline shared by the three orchestrators.

Reference stages (``ar_sparse_operation.py:289-362``): allocate tiled Q/K/V +
pools, copy padded text K/V, tile+pool Q and K/V (Triton), select blocks
(torch), block-sparse attention on the tiled tensors (Triton), untile. Here:

1. ``li_pool_blocks`` writes the q and k block means (normalised in the same
   launch for the cosine metric); the tiled copies are never materialised, and
   with a ``memory.KeyPoolCache`` only the changed key block rows are pooled;
2. ``li_select_blocks`` builds the sorted index list (text blocks first): a
   score kernel and a top-k kernel;
3. ``li_sparse_attn_raster`` reads q, the visual K/V and the text K/V straight
   from the caller's tensors, 3D block by 3D block, and writes the output in
   q's raster layout (plus a combine kernel when the last wave's tiles are
   split).

Four to six kernel launches (the key pooling is skipped when a key-pool cache
holds it; the combine runs only for a split tail), no host synchronisation, no
intermediate tiled tensors.
"""

from __future__ import annotations

import math
from typing import Optional

import torch

from . import _lib as L
from . import kernels as K


def latent_grids(q_len: int, k_len: int, latent_hw, tile):
    """Frame counts and block grids — ``ar_sparse_operation.py:319-327``."""
    LH, LW = latent_hw
    HW = LH * LW
    T_q, T_k = q_len // HW, k_len // HW
    return T_q, T_k, K.grid_blocks(T_q, LH, LW, tile), K.grid_blocks(T_k, LH, LW, tile)


def sparse_forward(q, k_txt, v_txt, k_vis, v_vis, latent_hw, params: dict, mode: int, default_tile,
                   default_metric: str = "cosine", ratio: Optional[float] = None, min_budget: int = 7,
                   q_block_offset: Optional[int] = None, score_bias: Optional[torch.Tensor] = None,
                   profile: Optional[dict] = None, out: Optional[torch.Tensor] = None, k_pool=None,
                   q_pool: Optional[torch.Tensor] = None):
    LH, LW = latent_hw
    tile = tuple(int(x) for x in params.get("tile_size", default_tile))
    text_len = k_txt.shape[2] if k_txt is not None else 0
    T_q, T_k, gq, gk = latent_grids(q.shape[2], k_vis.shape[2], latent_hw, tile)
    nq, nk = gq[0] * gq[1] * gq[2], gk[0] * gk[1] * gk[2]
    if mode == L.SELECT_BIDIR and q_block_offset is None and nq != nk:
        # generate_prefill_indices broadcasts an [N_k, N_k] neighbour matrix over
        # [.., N_q, N_k] scores and fails unless N_q == N_k.
        raise RuntimeError(f"bidirectional block selection needs N_q == N_k (got {nq} and {nk})")
    if k_vis.dtype != q.dtype:
        raise TypeError("q and k_vis must share a dtype")

    def mark(name):
        if profile is not None:
            ev = torch.cuda.Event(enable_timing=True)
            ev.record()
            profile[name] = ev

    metric = params.get("sim_metric", default_metric)
    # Cosine similarity is the plain dot product of the normalised pools (same
    # rounding chain); the pooling kernel normalises the rows it writes, which
    # keeps the normalisation out of the selection kernel's inner loop.
    cosine = metric == "cosine"
    mark("prep_start")
    if q_pool is not None:
        # Pooled by the caller (e.g. together with the key pool in one launch): the
        # block means of q, normalised for the cosine metric.
        if tuple(q_pool.shape) != (q.shape[0], q.shape[1], nq, q.shape[3]) or q_pool.dtype != q.dtype:
            raise ValueError("q_pool does not match this call's query grid")
    else:
        q_pool = K.pool_blocks(q, T_q, LH, LW, tile, normalized=cosine)
    if k_pool is not None:
        # memory.KeyPoolCache: the key pool was refreshed by the caller (only the
        # block rows whose frames changed were re-pooled).
        if k_pool.tile != tile or k_pool.pool is None or k_pool.pool.shape[2] != gk[0] * gk[1] * gk[2]:
            raise ValueError("k_pool cache does not match this call's key grid")
        key_pool = k_pool.selection_pool(metric)
    else:
        key_pool = K.pool_blocks(k_vis, T_k, LH, LW, tile, normalized=cosine)
    mark("prep_end")
    if cosine:
        metric = "dot"
    p = K.select_params(mode, metric, tile, gq, gk, text_len,
                        recent_protect=params.get("recent_protect", 0),
                        topk_ratio=params.get("topk_ratio", 1.0) if ratio is None else ratio,
                        min_budget=min_budget, q_block_offset=q_block_offset or 0)
    mark("index_start")
    idx, cnt = K.select_blocks(q_pool, key_pool, p, score_bias=score_bias)
    mark("index_end")
    mark("attn_start")
    out = K.sparse_attn_raster(q, L.grid3d(T_q, LH, LW, tile), k_txt, v_txt, k_vis, v_vis,
                               L.grid3d(T_k, LH, LW, tile), idx, cnt, sm_scale=1.0 / math.sqrt(q.shape[-1]),
                               out=out)
    mark("attn_end")
    return out


def dense_attention(q, k, v):
    """The reference's dense branch (``F.scaled_dot_product_attention``), kept
    where its orchestrators fall back to it (untileable query length; HY
    prefill warm-up chunks)."""
    return torch.nn.functional.scaled_dot_product_attention(q, k, v, dropout_p=0.0, is_causal=False)
