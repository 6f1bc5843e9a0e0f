"""Drop-in for HY-WorldPlay's ``ar_sparse_operation`` (autoregressive decode path).

Reference: hy-worldplay/files/hyvideo/models/transformers/modules/ar_sparse_operation.py.
Same public names and signatures; the Triton kernels and torch selection ops
are replaced by the sm_100a kernels of this package.
"""

from __future__ import annotations

import torch

from . import _lib as L
from . import kernels as K
from .pipeline import dense_attention, sparse_forward

#: The reference exposes ``HAS_TRITON`` to say whether its fused path is usable.
#: Here the fused path needs the native library; importing this module does not
#: load it, the first call does (and raises if it is missing).
HAS_TRITON = False
HAS_NATIVE = True

_DEFAULT_TILE = (4, 8, 4)  # ar_sparse_operation.py:319


def launch_q_prep(src, dst, mean, T, H, W, tt, th, tw, nh, nw):
    """Tile Q and write its block means — ``ar_sparse_operation.py:166-181``."""
    K.tile_pool(src, L.grid3d(T, H, W, (tt, th, tw)), dst0=dst, pool=mean)


def launch_kv_prep(k_src, v_src, k_dst, v_dst, k_mean, dst_off, pool_off, T, H, W, tt, th, tw, nh, nw):
    """Tile K and V after ``dst_off`` text blocks and write K's block means —
    ``ar_sparse_operation.py:183-202``."""
    K.tile_pool(k_src, L.grid3d(T, H, W, (tt, th, tw)), src1=v_src, dst0=k_dst, dst1=v_dst,
                dst_block_offset=dst_off, pool=k_mean, pool_block_offset=pool_off)


def launch_untile(src, dst, T, H, W, tt, th, tw, nh, nw):
    """Tiled output back to raster order — ``ar_sparse_operation.py:204-218``."""
    K.untile(src, dst, L.grid3d(T, H, W, (tt, th, tw)))


def fast_generate_indices(q_pool, k_pool, text_len, grid_thw_q, grid_thw_k, params, device):
    """Decode block selection — ``ar_sparse_operation.py:223-284``.

    Returns ``(final_indices, final_counts)``: int32 ``[B, H, Nq_blk, ntxt + k]``
    (text blocks ``0..ntxt-1`` first, then the selected visual blocks offset by
    ``ntxt``, ascending) and int32 counts ``[B, H, Nq_blk]``.
    """
    p = K.select_params(L.SELECT_DECODE, params.get("sim_metric", "cosine"), params["tile_size"], grid_thw_q,
                        grid_thw_k, text_len, recent_protect=params.get("recent_protect", 0),
                        topk_ratio=params.get("topk_ratio", 1.0))
    return K.select_blocks(q_pool, k_pool, p)


def run_sparse_attention(q, k_txt, v_txt, k_vis, v_vis, block_idx, latent_hw, sparse_params):
    """One autoregressive sparse-attention forward — ``ar_sparse_operation.py:289-362``.

    q ``[B, H, Nq, D]``, text K/V ``[B, H, N_txt, D]``, visual K/V ``[B, H, N_vis, D]``
    (any strides with D contiguous). Falls back to dense attention, as the
    reference does, when the query length is not a whole number of latent frames.
    Device-side errors (a bounded wait that gave up; a block id out of range)
    do not raise here: the kernels record them in the device error word, which
    ``kernels.raise_device_errors()`` reads (and synchronises) at a step boundary.
    """
    LH, LW = latent_hw
    if q.shape[2] % (LH * LW) != 0:
        return dense_attention(q, torch.cat([k_txt, k_vis], dim=2), torch.cat([v_txt, v_vis], dim=2))
    return sparse_forward(q, k_txt, v_txt, k_vis, v_vis, latent_hw, sparse_params, L.SELECT_DECODE,
                          _DEFAULT_TILE)
