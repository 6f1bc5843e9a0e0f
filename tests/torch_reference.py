"""The reference's block selection as it runs in production: torch ops on CUDA tensors
(test infrastructure, used only to measure how often the library's exactly rounded
selection differs from the reference's own GPU arithmetic, and why).

The patched HY-WorldPlay and Matrix-Game-3.0 pipelines call the selection with CUDA
tensors, so the block-score GEMM is a cuBLAS bf16 matmul with fp32 accumulation in
cuBLAS's order and ``torch.topk`` / ``torch.sort`` are torch's CUDA kernels. This module
restates those op sequences on torch tensors:

* decode: ``ar_sparse_operation.py:223-284`` (``fast_generate_indices``);
* bidirectional: ``bi_sparse_operation.py:179-234`` and
  ``bi_sparse_operation_for_KV_cache.py:220-296`` (``generate_prefill_indices``),
  which needs a square score matrix.

Both return the ranking scores handed to ``torch.topk`` and the sorted visual block
indices (before the text offset).
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F

LARGE_BIAS = 1e6


def _similarity(q_pool: torch.Tensor, k_pool: torch.Tensor, metric: str) -> torch.Tensor:
    """``sim`` of ``ar_sparse_operation.py:250-256`` / ``bi_sparse_operation.py:195-201``."""
    if metric == "cosine":
        return torch.matmul(F.normalize(q_pool, dim=-1), F.normalize(k_pool, dim=-1).transpose(-2, -1))
    sim = torch.matmul(q_pool, k_pool.transpose(-2, -1))
    if metric == "scaled_dot_product":
        sim = sim * (1.0 / math.sqrt(q_pool.shape[-1]))
    return sim


def decode_select(q_pool, k_pool, tile, grid_q, params):
    """Ranking scores and sorted visual indices of the decode selection."""
    tt = tile[0]
    nk = k_pool.shape[2]
    rank = _similarity(q_pool, k_pool, params.get("sim_metric", "cosine")).clone()
    n_prot = 0
    rp = params.get("recent_protect", 0)
    if rp > 0:
        n_prot = min(((rp + tt - 1) // tt) * grid_q[1] * grid_q[2], nk)
        if n_prot > 0:
            rank[..., -n_prot:] += LARGE_BIAS
    k = n_prot + int(max(0, nk - n_prot) * params.get("topk_ratio", 1.0))
    k = min(max(k, 1 if nk > 0 else 0), nk)
    _, idx = torch.topk(rank, k=k, dim=-1)
    idx, _ = torch.sort(idx, dim=-1)
    return rank, idx


def bidir_select(q_pool, k_pool, grid_k, params):
    """Ranking scores and sorted visual indices of the bidirectional selection
    (square: ``q_pool`` has one row per key block)."""
    sim = _similarity(q_pool, k_pool, params.get("sim_metric", "cosine"))
    nk = sim.shape[-1]
    _, Nh, Nw = grid_k
    ar = torch.arange(nk, device=sim.device)
    t, rem = ar // (Nh * Nw), ar % (Nh * Nw)
    h, w = rem // Nw, rem % Nw
    dist = ((t[:, None] - t[None, :]).abs() + (h[:, None] - h[None, :]).abs()
            + (w[:, None] - w[None, :]).abs())
    rank = sim.clone() + (dist <= 1).to(sim.dtype) * LARGE_BIAS
    k = min(max(int(nk * params.get("topk_ratio", 0.25)), 7), nk)
    _, idx = torch.topk(rank, k=k, dim=-1)
    idx, _ = torch.sort(idx, dim=-1)
    return rank, idx
