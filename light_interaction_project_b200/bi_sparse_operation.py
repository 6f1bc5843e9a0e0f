"""Drop-in for Matrix-Game-3.0's ``wan.modules.bi_sparse_operation``.

Reference: matrix-game-3.0/files/wan/modules/bi_sparse_operation.py.
"""

from __future__ import annotations

import torch

from . import _lib as L
from . import kernels as K
from .ar_sparse_operation import launch_kv_prep, launch_q_prep, launch_untile  # noqa: F401  (same surface)
from .bi_sparse_operation_for_KV_cache import _pools
from .pipeline import dense_attention, sparse_forward

#: Stage profiler switch (``bi_sparse_operation.py:13``): when True every call
#: records CUDA events around selection prep, indexing and attention and prints
#: a per-stage line (this synchronises, so keep it off in production).
ENABLE_SPARSE_PROFILING = False
HAS_TRITON = False
HAS_NATIVE = True

_DEFAULT_TILE = (4, 4, 8)  # bi_sparse_operation.py:253


def generate_prefill_indices(q_in, k_in, text_len, grid_thw, params, device, q_block_offset=None):
    """Bidirectional block selection — ``bi_sparse_operation.py:179-234``
    (``topk_ratio`` defaults to 0.25 here, as in the reference)."""
    q_pool, bs = _pools(q_in, params)
    k_pool, _ = _pools(k_in, params)
    nq, nk = q_pool.shape[2], k_pool.shape[2]
    if q_block_offset is None and nq != nk:
        raise RuntimeError(f"bidirectional block selection needs N_q == N_k (got {nq} and {nk})")
    tile = (1, 1, bs) if q_in.dim() == 5 else params["tile_size"]
    p = K.select_params(L.SELECT_BIDIR, params.get("sim_metric", "cosine"), tile, grid_thw, grid_thw, text_len,
                        topk_ratio=params.get("topk_ratio", 0.25), min_budget=7,
                        q_block_offset=q_block_offset or 0)
    return K.select_blocks(q_pool, k_pool, p)


def run_sparse_attention(q, k, v, text_len, block_idx, latent_hw, sparse_params, q_block_offset=None, out=None,
                         k_pool=None, q_pool=None):
    """One Matrix-Game sparse-attention forward — ``bi_sparse_operation.py:236-348``.

    ``k``/``v`` hold ``text_len`` text tokens followed by the visual tokens. Dense
    when the query length is not a whole number of latent frames.
    ``q_block_offset`` (extension): q covers only the last query-chunk frames of
    the key sequence; the selection then equals those rows of the full
    bidirectional selection.
    ``out`` (extension): a tensor shaped like q, any strides the attention's
    store map can describe (D contiguous, 16-byte strides), that receives the
    output — e.g. a ``[B, S, H, D]`` buffer seen as ``[B, H, S, D]``, so the
    output projection reads it without a re-layout copy.
    ``k_pool`` (extension): a ``memory.KeyPoolCache`` refreshed by the caller for
    this ``k``'s visual part; the key pooling is then skipped.
    ``q_pool`` (extension): q's block means ``[B, H, Nq_blk, D]`` computed by the
    caller (normalised for the cosine metric), e.g. in the same
    ``kernels.pool_blocks_multi`` launch as the key pool; the q pooling is then
    skipped.
    Device-side errors (a bounded wait that gave up; a block id out of range)
    do not raise here: the kernels record them in the device error word, which
    ``kernels.raise_device_errors()`` reads (and synchronises) at a step boundary.
    """
    LH, LW = latent_hw
    if q.shape[2] % (LH * LW) != 0:
        o = dense_attention(q, k, v)
        if out is not None:
            out.copy_(o)
            o = out
        return o
    prof = {} if ENABLE_SPARSE_PROFILING else None
    if prof is not None:
        start = torch.cuda.Event(enable_timing=True)
        start.record()
    out = sparse_forward(q, k[:, :, :text_len], v[:, :, :text_len], k[:, :, text_len:], v[:, :, text_len:],
                         latent_hw, sparse_params, L.SELECT_BIDIR, _DEFAULT_TILE,
                         ratio=sparse_params.get("topk_ratio", 0.25), q_block_offset=q_block_offset, profile=prof,
                         out=out, k_pool=k_pool, q_pool=q_pool)
    if prof is not None:
        torch.cuda.synchronize()
        t = lambda a, b: prof[a].elapsed_time(prof[b])  # noqa: E731
        print(f"[Block {block_idx:2d}] Sparse Workflow: Total {start.elapsed_time(prof['attn_end']):>5.2f}ms | "
              f"Pool {t('prep_start', 'prep_end'):>4.2f}ms | Index {t('index_start', 'index_end'):>4.2f}ms | "
              f"SparseAttn+Untile {t('attn_start', 'attn_end'):>4.2f}ms")
    return out
