"""CPU restatement of the reference's block-sparse attention path (test infrastructure).

Every function states the reference lines it follows. Paths are relative to the
reference project root (2843721358l-del/Light-Interaction-Project).

Arrays are numpy float32 holding values exactly representable in the working
dtype ('bf16' or 'fp32'), or int32 for indices. Layouts follow the reference:
raster ``[B, H, L, D]`` with ``L = T * LH * LW`` in (t, h, w) order, tiled
``[B, H, Nblk, bs, D]`` with blocks in (nt, nh, nw) order and tokens inside a
block in (tt, th, tw) order (``ar_sparse_operation.py:42-52``).

Rounding rules (the contract the CUDA kernels reproduce bit for bit)
-------------------------------------------------------------------
The reference accumulates in fp32 in an order set by Triton, cuBLAS or MKL, and
then rounds to the input dtype. That order differs between CPU and GPU. This
restatement fixes one deterministic order whose fp32 result is, in practice,
the correctly rounded exact value:

* block mean (``ar_sparse_operation.py:69-70``): eight interleaved fp64
  partial sums ``p_g = sum_i x[8i+g]`` (sequential in i), combined
  ``((p0+p1)+p2)+...+p7`` in fp64, rounded to fp32, divided by ``fp32(bs)`` in
  fp32, rounded to the dtype (RNE).
* dot products in the block-score GEMM (``ar_sparse_operation.py:252-256``):
  exact products summed in fp64 as four interleaved partial sums over d
  (``p_g = sum_i x[4i+g]``, combined ``((p0+p1)+p2)+p3``), rounded to fp32,
  then to the dtype.
* ``F.normalize``: sum of squares as a dot product above, fp32 ``sqrt``,
  rounded to the dtype, clamped below at ``dtype(1e-12)``, then the
  element-wise fp32 quotient rounded to the dtype.
* scalar multiply / add on a dtype tensor (``* (1/sqrt(d))``, ``+= 1e6``):
  one fp32 operation with the scalar converted to fp32, rounded to the dtype
  (torch's opmath rule for reduced-precision tensors).
* top-k ranks by torch's radix order of the dtype's bit pattern (so -0.0 ranks
  below +0.0) and resolves ties at the k-th value lowest index first, as
  torch's CUDA top-k does.
"""

from __future__ import annotations

import math
from typing import Dict, Sequence, Tuple

import numpy as np

__all__ = [
    "round_to", "bf16_bits", "radix_key", "grid_dims", "tile_raster", "untile_raster",
    "block_mean", "tile_pool", "normalize_rows", "block_scores", "select_topk",
    "fast_generate_indices", "generate_prefill_indices", "decode_budget",
    "prefill_budget", "sparse_attention_tiled", "dense_masked_attention",
    "gather_frames", "run_sparse_attention_hy", "run_sparse_attention_mg",
    "run_sparse_prefill_attention_hy",
]

LARGE_BIAS = 1e6


# ----------------------------------------------------------------------------
# Rounding helpers
# ----------------------------------------------------------------------------
def round_to(x, dtype: str) -> np.ndarray:
    """Round float32 values to ``dtype`` with round-to-nearest-even."""
    x = np.ascontiguousarray(np.asarray(x, dtype=np.float32))
    if dtype == "fp32":
        return x
    if dtype == "fp16":
        with np.errstate(over="ignore"):  # overflow to inf, as the GPU conversion does
            return x.astype(np.float16).astype(np.float32)
    if dtype != "bf16":
        raise ValueError(f"unsupported dtype {dtype}")
    u = x.view(np.uint32).astype(np.uint64)
    r = ((u + np.uint64(0x7FFF) + ((u >> np.uint64(16)) & np.uint64(1))) & np.uint64(0xFFFF0000))
    out = r.astype(np.uint32).view(np.float32).copy()
    nan = np.isnan(x)
    if nan.any():
        out[nan] = np.nan
    return out


def bf16_bits(x: np.ndarray) -> np.ndarray:
    """uint16 bit patterns of bf16-representable float32 values."""
    return (np.ascontiguousarray(x, dtype=np.float32).view(np.uint32) >> 16).astype(np.uint16)


def radix_key(x: np.ndarray, dtype: str) -> np.ndarray:
    """Order-preserving unsigned key (torch's TopKTypeConfig transform; NaN highest)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    if dtype in ("bf16", "fp16"):
        if dtype == "bf16":
            b = bf16_bits(x).astype(np.uint32)
        else:
            b = x.astype(np.float16).view(np.uint16).astype(np.uint32)
        key = np.where(b & 0x8000, b ^ 0xFFFF, b ^ 0x8000)
        return np.where(np.isnan(x), 0xFFFF, key).astype(np.uint64)
    b = x.view(np.uint32).astype(np.uint64)
    key = np.where(b & 0x80000000, b ^ 0xFFFFFFFF, b ^ 0x80000000)
    return np.where(np.isnan(x), 0xFFFFFFFF, key).astype(np.uint64)


# ----------------------------------------------------------------------------
# 3D tiling, pooling, untiling
# ----------------------------------------------------------------------------
def grid_dims(T: int, LH: int, LW: int, tile: Sequence[int]) -> Tuple[int, int, int]:
    """Block grid ``(nt, nh, nw)`` — ``ar_sparse_operation.py:322-324``."""
    tt, th, tw = tile
    return (T + tt - 1) // tt, (LH + th - 1) // th, (LW + tw - 1) // tw


def _block_token_index(T, LH, LW, tile):
    """Raster token index per (block, in-block token), -1 for padding.

    Mirrors the coordinate arithmetic of ``_fused_q_prep_kernel``
    (``ar_sparse_operation.py:41-59``).
    """
    tt, th, tw = tile
    nt, nh, nw = grid_dims(T, LH, LW, tile)
    blk = np.arange(nt * nh * nw)
    cur_nw = blk % nw
    cur_nh = (blk // nw) % nh
    cur_nt = blk // (nw * nh)
    off = np.arange(tt * th * tw)
    o_tw = off % tw
    o_th = (off // tw) % th
    o_tt = off // (tw * th)
    ct = cur_nt[:, None] * tt + o_tt[None, :]
    ch = cur_nh[:, None] * th + o_th[None, :]
    cw = cur_nw[:, None] * tw + o_tw[None, :]
    valid = (ct < T) & (ch < LH) & (cw < LW)
    idx = ct * (LH * LW) + ch * LW + cw
    return np.where(valid, idx, -1)


def tile_raster(x: np.ndarray, T: int, LH: int, LW: int, tile) -> np.ndarray:
    """Raster ``[B,H,T*LH*LW,D]`` -> tiled ``[B,H,Nblk,bs,D]`` with zero fill.

    ``_fused_q_prep_kernel`` store half (``ar_sparse_operation.py:62-66``).
    """
    B, H, L, D = x.shape
    if L < T * LH * LW:
        raise ValueError("raster length shorter than T*LH*LW")
    tok = _block_token_index(T, LH, LW, tile)
    src = np.concatenate([x, np.zeros((B, H, 1, D), x.dtype)], axis=2)
    gather = np.where(tok >= 0, tok, L)
    return src[:, :, gather, :]


def untile_raster(o_tiled: np.ndarray, T: int, LH: int, LW: int, tile) -> np.ndarray:
    """Tiled -> raster, dropping padded rows (``ar_sparse_operation.py:127-161``)."""
    B, H, nblk, bs, D = o_tiled.shape
    tok = _block_token_index(T, LH, LW, tile)
    out = np.zeros((B, H, T * LH * LW, D), o_tiled.dtype)
    valid = tok >= 0
    out[:, :, tok[valid], :] = o_tiled[:, :, valid, :]
    return out


def block_mean(tiled: np.ndarray, dtype: str) -> np.ndarray:
    """Per-block mean (``ar_sparse_operation.py:69-70``; ``:121-122``) with the fixed
    eight-way interleaved fp64 order described in the module docstring."""
    bs = tiled.shape[-2]
    if bs % 8:
        raise ValueError("block size must be a multiple of 8")
    t64 = tiled.astype(np.float64)
    total = None
    for g in range(8):
        acc = np.zeros(t64.shape[:-2] + t64.shape[-1:], np.float64)
        for i in range(g, bs, 8):
            acc = acc + t64[..., i, :]
        total = acc if total is None else total + acc
    mean = total.astype(np.float32) / np.float32(bs)
    return round_to(mean.astype(np.float32), dtype)


def tile_pool(x: np.ndarray, T: int, LH: int, LW: int, tile, dtype: str):
    """Fused tile + mean pool (``launch_q_prep`` / ``launch_kv_prep``,
    ``ar_sparse_operation.py:166-202``). Returns ``(tiled, pool)``."""
    tiled = tile_raster(x, T, LH, LW, tile)
    return tiled, block_mean(tiled, dtype)


# ----------------------------------------------------------------------------
# Block selection
# ----------------------------------------------------------------------------
def _sum4(prod):
    """Fixed-order fp64 sum over the last axis: four interleaved partial sums
    ``p_g = sum_i x[4i+g]`` (sequential in i), combined ``((p0+p1)+p2)+p3``."""
    D = prod.shape[-1]
    parts = []
    for g in range(4):
        acc = np.zeros(prod.shape[:-1], np.float64)
        for d in range(g, D, 4):
            acc = acc + prod[..., d]
        parts.append(acc)
    return ((parts[0] + parts[1]) + parts[2]) + parts[3]


def _dot_rows(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """fp64 dot products ``a[..., i, :] . b[..., j, :]`` of exact products in the
    :func:`_sum4` order, rounded to fp32."""
    a64 = a.astype(np.float64)
    b64 = b.astype(np.float64)
    D = a.shape[-1]
    parts = []
    for g in range(4):
        acc = np.zeros(a.shape[:-1] + (b.shape[-2],), np.float64)
        for d in range(g, D, 4):
            acc = acc + a64[..., :, None, d] * b64[..., None, :, d]
        parts.append(acc)
    return (((parts[0] + parts[1]) + parts[2]) + parts[3]).astype(np.float32)


def normalize_rows(p: np.ndarray, dtype: str) -> np.ndarray:
    """``F.normalize(p, dim=-1)`` on a ``dtype`` tensor (``ar_sparse_operation.py:252``)."""
    p64 = p.astype(np.float64)
    ss = _sum4(p64 * p64)
    nrm = round_to(np.sqrt(ss.astype(np.float32)), dtype)
    eps = round_to(np.float32(1e-12), dtype)
    den = np.maximum(nrm, eps)
    return round_to((p / den[..., None]).astype(np.float32), dtype)


def block_scores(q_pool: np.ndarray, k_pool: np.ndarray, metric: str, dtype: str) -> np.ndarray:
    """Block similarity ``sim`` (``ar_sparse_operation.py:250-256``;
    ``bi_sparse_operation.py:195-201``)."""
    d = q_pool.shape[-1]
    if metric == "cosine":
        qn = normalize_rows(q_pool, dtype)
        kn = normalize_rows(k_pool, dtype)
        return round_to(_dot_rows(qn, kn), dtype)
    sim = round_to(_dot_rows(q_pool, k_pool), dtype)
    if metric == "scaled_dot_product":
        sim = round_to((sim * np.float32(1.0 / math.sqrt(d))).astype(np.float32), dtype)
    return sim


def select_topk(score: np.ndarray, k: int, dtype: str) -> np.ndarray:
    """Indices of the ``k`` largest scores per row, sorted ascending.

    Rank by radix key descending; ties at the k-th value go to the lowest
    index (``torch.topk`` on CUDA followed by ``torch.sort``,
    ``ar_sparse_operation.py:274-276``).
    """
    nk = score.shape[-1]
    if k == 0:
        return np.zeros(score.shape[:-1] + (0,), np.int64)
    key = radix_key(score, dtype)
    # Composite key: high part = radix key, low part = reversed index. Unique.
    comp = (key << np.uint64(32)) | (np.uint64(0xFFFFFFFF) - np.arange(nk, dtype=np.uint64))
    order = np.argsort(comp, axis=-1, kind="stable")
    top = order[..., nk - k:]
    return np.sort(top, axis=-1)


def decode_budget(nk: int, tile, grid_thw_q, params: Dict) -> Tuple[int, int]:
    """``(n_prot_blk, k_budget)`` of ``fast_generate_indices``
    (``ar_sparse_operation.py:260-272``)."""
    tt = tile[0]
    Nh, Nw = grid_thw_q[1], grid_thw_q[2]
    n_prot = 0
    rp = params.get("recent_protect", 0)
    if rp > 0:
        n_prot = min(((rp + tt - 1) // tt) * Nh * Nw, nk)
    n_hist = max(0, nk - n_prot)
    k_hist = int(n_hist * params.get("topk_ratio", 1.0))
    k = n_prot + k_hist
    k = min(max(k, 1 if nk > 0 else 0), nk)
    return n_prot, k


def prefill_budget(nk: int, ratio: float) -> int:
    """``k_budget`` of ``generate_prefill_indices``
    (``bi_sparse_operation_for_KV_cache.py:282-285``)."""
    return min(max(int(nk * ratio), 7), nk)


def _add_scalar(x, s, dtype):
    return round_to((x.astype(np.float32) + np.float32(s)).astype(np.float32), dtype)


def _finish(vis_idx: np.ndarray, text_len: int, bs: int):
    ntxt = (text_len + bs - 1) // bs
    B, H, Nq, _ = vis_idx.shape
    txt = np.broadcast_to(np.arange(ntxt, dtype=np.int64), (B, H, Nq, ntxt))
    idx = np.concatenate([txt, vis_idx + ntxt], axis=-1).astype(np.int32)
    cnt = np.full((B, H, Nq), idx.shape[-1], np.int32)
    return np.ascontiguousarray(idx), cnt


def _with_bias(sim, score_bias, dtype):
    """Additive score bias (harness extension, no reference counterpart): one
    fp32 add rounded to the dtype, before the protection bias — the selection
    kernels' ``score_bias`` input."""
    if score_bias is None:
        return sim
    b = np.broadcast_to(np.asarray(score_bias, np.float32), sim.shape)
    return round_to((sim.astype(np.float32) + b).astype(np.float32), dtype)


def fast_generate_indices(q_pool, k_pool, text_len, grid_thw_q, grid_thw_k, params, dtype,
                          return_scores=False, score_bias=None):
    """Decode-path selection — ``ar_sparse_operation.py:223-284``."""
    tile = params["tile_size"]
    bs = tile[0] * tile[1] * tile[2]
    nk = k_pool.shape[2]
    sim = _with_bias(block_scores(q_pool, k_pool, params.get("sim_metric", "cosine"), dtype), score_bias, dtype)
    rank = sim.copy()
    n_prot, k = decode_budget(nk, tile, grid_thw_q, params)
    if n_prot > 0:
        rank[..., nk - n_prot:] = _add_scalar(rank[..., nk - n_prot:], LARGE_BIAS, dtype)
    vis = select_topk(rank, k, dtype)
    idx, cnt = _finish(vis, text_len, bs)
    return (idx, cnt, rank) if return_scores else (idx, cnt)


def _neighbor_matrix(nq, nk, grid_thw, q_offset=0):
    _, Nh, Nw = grid_thw
    kk = np.arange(nk)
    qq = np.arange(nq) + q_offset
    tq, hq, wq = qq // (Nh * Nw), (qq % (Nh * Nw)) // Nw, qq % Nw
    tk, hk, wk = kk // (Nh * Nw), (kk % (Nh * Nw)) // Nw, kk % Nw
    dist = (np.abs(tq[:, None] - tk[None, :]) + np.abs(hq[:, None] - hk[None, :])
            + np.abs(wq[:, None] - wk[None, :]))
    return dist <= 1


def generate_prefill_indices(q_pool, k_pool, text_len, grid_thw, params, dtype,
                             q_offset=None, return_scores=False, score_bias=None):
    """Bidirectional selection — ``bi_sparse_operation_for_KV_cache.py:220-296``,
    ``bi_sparse_operation.py:179-234``.

    The reference needs ``N_q == N_k`` (the neighbour matrix is ``[N_k, N_k]``).
    ``q_offset`` (block offset of query row 0 in the key grid) computes a subset of
    the rows of that square problem; rows are independent, so the result equals
    the matching rows of the full selection. ``None`` requires ``N_q == N_k``.
    """
    tile = params["tile_size"]
    bs = tile[0] * tile[1] * tile[2]
    nq, nk = q_pool.shape[2], k_pool.shape[2]
    if q_offset is None:
        if nq != nk:
            raise RuntimeError(f"bidirectional selection needs N_q == N_k (got {nq} and {nk})")
        q_offset = 0
    if q_offset < 0 or q_offset + nq > nk:
        raise ValueError("query rows outside the key grid")
    sim = _with_bias(block_scores(q_pool, k_pool, params.get("sim_metric", "cosine"), dtype), score_bias, dtype)
    bias = round_to(np.float32(1.0) * np.float32(LARGE_BIAS), dtype)
    nb = _neighbor_matrix(nq, nk, grid_thw, q_offset)
    rank = round_to((sim + np.where(nb, bias, np.float32(0.0))).astype(np.float32), dtype)
    k = prefill_budget(nk, params.get("topk_ratio", 0.25))
    vis = select_topk(rank, k, dtype)
    idx, cnt = _finish(vis, text_len, bs)
    return (idx, cnt, rank) if return_scores else (idx, cnt)


# ----------------------------------------------------------------------------
# Attention
# ----------------------------------------------------------------------------
def sparse_attention_tiled(q_tiled, k_all, v_all, indices, counts, sm_scale=None,
                           p_dtype=None):
    """Block-sparse attention over tiled tensors (fp32 math).

    Semantics of ``_attn_fwd_bsa_align`` (``longcat_kernel.py`` HY ``:100-155``)
    with every query block using its own index list: query block ``i`` attends to
    the ``counts[i]`` key blocks ``indices[i, :counts[i]]``; padded (zero) key rows
    take part in the softmax. ``p_dtype='bf16'`` rounds the probabilities to bf16
    before the PV product, as the reference kernel does (``:141``).
    Returns ``(o_tiled, lse_log2)``.
    """
    import torch
    q = torch.from_numpy(np.ascontiguousarray(q_tiled, np.float32))
    k = torch.from_numpy(np.ascontiguousarray(k_all, np.float32))
    v = torch.from_numpy(np.ascontiguousarray(v_all, np.float32))
    B, H, nq, bs, D = q.shape
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(D)
    o = torch.zeros_like(q)
    lse = torch.full((B, H, nq, bs), float("-inf"))
    idx = np.asarray(indices)
    cnt = np.asarray(counts)
    for b in range(B):
        for h in range(H):
            for c in np.unique(cnt[b, h]):
                rows = np.nonzero(cnt[b, h] == c)[0]
                if c == 0:
                    continue
                sel = torch.from_numpy(idx[b, h][rows][:, :c].astype(np.int64))
                ks = k[b, h][sel].reshape(len(rows), c * bs, D)
                vs = v[b, h][sel].reshape(len(rows), c * bs, D)
                qs = q[b, h][torch.from_numpy(rows)]
                s = torch.bmm(qs, ks.transpose(1, 2)) * sm_scale
                m = s.amax(dim=-1, keepdim=True)
                p = torch.exp(s - m)
                l = p.sum(-1, keepdim=True)
                if p_dtype == "bf16":
                    p = p.to(torch.bfloat16).to(torch.float32)
                o[b, h, torch.from_numpy(rows)] = torch.bmm(p, vs) / l
                lse[b, h, torch.from_numpy(rows)] = ((m + torch.log(l)) / math.log(2)).squeeze(-1)
    return o.numpy(), lse.numpy()


def dense_masked_attention(q_tiled, k_all, v_all, indices, counts, sm_scale=None, threads=None):
    """Dense masked attention applying the block mask (the reference's CPU path).

    Scores against every key block, mask to the selected ones, softmax, PV —
    ``scaled_dot_product_attention`` with a boolean block mask, one head at a
    time. Same result as :func:`sparse_attention_tiled`; this is the form timed
    as the CPU baseline.
    """
    import torch
    if threads:
        torch.set_num_threads(threads)
    q = torch.as_tensor(q_tiled, dtype=torch.float32)
    k = torch.as_tensor(k_all, dtype=torch.float32)
    v = torch.as_tensor(v_all, dtype=torch.float32)
    B, H, nq, bs, D = q.shape
    nkb = k.shape[2]
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(D)
    out = torch.empty_like(q)
    idx = torch.as_tensor(np.asarray(indices, np.int64))
    cnt = torch.as_tensor(np.asarray(counts, np.int64))
    for b in range(B):
        for h in range(H):
            blk_mask = torch.zeros(nq, nkb, dtype=torch.bool)
            ar = torch.arange(idx.shape[-1])
            valid = ar[None, :] < cnt[b, h][:, None]
            rows = torch.arange(nq)[:, None].expand_as(idx[b, h])
            blk_mask[rows[valid], idx[b, h][valid]] = True
            mask = blk_mask.repeat_interleave(bs, 0).repeat_interleave(bs, 1)
            o = torch.nn.functional.scaled_dot_product_attention(
                q[b, h].reshape(1, nq * bs, D), k[b, h].reshape(1, nkb * bs, D),
                v[b, h].reshape(1, nkb * bs, D), attn_mask=mask[None], scale=sm_scale)
            out[b, h] = o.reshape(nq, bs, D)
    return out.numpy()


# ----------------------------------------------------------------------------
# Memory-pruning gather
# ----------------------------------------------------------------------------
def gather_frames(pool: np.ndarray, frame_ids, frame_tokens: int) -> np.ndarray:
    """Keep retained frames in the given order: ``pool[:, :, frames]`` on a
    ``[B, H, F*HW, D]`` K/V pool (``hy patch:3213-3221`` latent gather,
    ``mg patch:447-457``)."""
    B, H, L, D = pool.shape
    F = L // frame_tokens
    fr = pool.reshape(B, H, F, frame_tokens, D)
    return fr[:, :, np.asarray(frame_ids, np.int64)].reshape(B, H, -1, D)


# ----------------------------------------------------------------------------
# Orchestrators (restated end-to-end; raster in, raster out)
# ----------------------------------------------------------------------------
def _text_blocks(k_txt, bs):
    B, H, n, D = k_txt.shape
    ntxt = (n + bs - 1) // bs
    pad = ntxt * bs - n
    if pad:
        k_txt = np.concatenate([k_txt, np.zeros((B, H, pad, D), k_txt.dtype)], axis=2)
    return k_txt.reshape(B, H, ntxt, bs, D)


def _orchestrate(q, k_txt, v_txt, k_vis, v_vis, latent_hw, params, dtype, mode, q_offset=None):
    LH, LW = latent_hw
    tile = tuple(params["tile_size"])
    bs = tile[0] * tile[1] * tile[2]
    T_q = q.shape[2] // (LH * LW)
    T_k = k_vis.shape[2] // (LH * LW)
    q_t, q_p = tile_pool(q, T_q, LH, LW, tile, dtype)
    k_t, k_p = tile_pool(k_vis, T_k, LH, LW, tile, dtype)
    v_t = tile_raster(v_vis, T_k, LH, LW, tile)
    text_len = k_txt.shape[2]
    k_all = np.concatenate([_text_blocks(k_txt, bs), k_t], axis=2)
    v_all = np.concatenate([_text_blocks(v_txt, bs), v_t], axis=2)
    gq = grid_dims(T_q, LH, LW, tile)
    gk = grid_dims(T_k, LH, LW, tile)
    if mode == "decode":
        idx, cnt = fast_generate_indices(q_p, k_p, text_len, gq, gk, params, dtype)
    else:
        idx, cnt = generate_prefill_indices(q_p, k_p, text_len, gk, params, dtype, q_offset=q_offset)
    o_t, _ = sparse_attention_tiled(q_t, k_all, v_all, idx, cnt)
    o = untile_raster(o_t, T_q, LH, LW, tile)
    return round_to(o, dtype), dict(q_pool=q_p, k_pool=k_p, indices=idx, counts=cnt)


def run_sparse_attention_hy(q, k_txt, v_txt, k_vis, v_vis, latent_hw, params, dtype):
    """HY decode orchestrator (``ar_sparse_operation.py:289-362``), sparse branch."""
    return _orchestrate(q, k_txt, v_txt, k_vis, v_vis, latent_hw, params, dtype, "decode")


def run_sparse_prefill_attention_hy(q, k_txt, v_txt, k_vis, v_vis, latent_hw, params, dtype,
                                    q_offset=None):
    """HY prefill orchestrator (``bi_sparse_operation_for_KV_cache.py:301-395``), sparse branch."""
    return _orchestrate(q, k_txt, v_txt, k_vis, v_vis, latent_hw, params, dtype, "bidir", q_offset)


def run_sparse_attention_mg(q, k, v, text_len, latent_hw, params, dtype, q_offset=None):
    """MG orchestrator (``bi_sparse_operation.py:236-348``), sparse branch."""
    return _orchestrate(q, k[:, :, :text_len], v[:, :, :text_len], k[:, :, text_len:],
                        v[:, :, text_len:], latent_hw, params, dtype, "bidir", q_offset)
