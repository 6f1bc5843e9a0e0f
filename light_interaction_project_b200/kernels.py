"""Torch-facing wrappers of the CUDA kernels (one function per C-ABI entry point).

All outputs are allocated here with torch's caching allocator (the C ABI never
allocates) and every launch goes on the current CUDA stream. No host
synchronisation happens on these paths; device-side error bits (bad index,
bounded-wait timeout) accumulate in a per-device error word that
:func:`device_errors` reads (that read synchronises).
"""

from __future__ import annotations

import math
from typing import Optional, Sequence, Tuple

import torch

from . import _lib as L

_err_words = {}


def error_word(device) -> torch.Tensor:
    """Per-device int32 word the kernels OR error bits into."""
    dev = torch.device(device)
    key = dev.index if dev.index is not None else torch.cuda.current_device()
    w = _err_words.get(key)
    if w is None:
        w = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", key))
        _err_words[key] = w
    return w


def device_errors(device=None, clear: bool = True) -> int:
    """Synchronises and returns the accumulated device error bits."""
    w = error_word(device if device is not None else torch.cuda.current_device())
    v = int(w.item())
    if clear and v:
        w.zero_()
    return v


def raise_device_errors(device=None):
    v = device_errors(device)
    if v & L.LI_DEVERR_TIMEOUT:
        raise RuntimeError("li_b200: a device-side wait timed out")
    if v & L.LI_DEVERR_BAD_INDEX:
        raise ValueError("li_b200: an index (block id or frame id) was out of bounds")
    if v & L.LI_DEVERR_RANGE:
        raise ValueError("li_b200: an fp32 attention operand exceeded the fp16 range (|x| > 65504) of the fp32 path")


def grid_blocks(T: int, LH: int, LW: int, tile: Sequence[int]) -> Tuple[int, int, int]:
    tt, th, tw = tile
    return (T + tt - 1) // tt, (LH + th - 1) // th, (LW + tw - 1) // tw


def tile_pool(src0: torch.Tensor, grid: L.Grid3d, *, src1: Optional[torch.Tensor] = None,
              frame_ids: Optional[torch.Tensor] = None, dst0: Optional[torch.Tensor] = None,
              dst1: Optional[torch.Tensor] = None, dst_block_offset: int = 0,
              pool: Optional[torch.Tensor] = None, pool_block_offset: int = 0):
    """Tile (and/or mean-pool) one or two raster streams — ``li_tile_pool``."""
    lib = L.load()
    v0 = L.view4(src0, "src0")
    v1 = L.view4(src1, "src1") if src1 is not None else None
    d0 = L.view5(dst0, "dst0") if dst0 is not None else None
    d1 = L.view5(dst1, "dst1") if dst1 is not None else None
    pv = L.view4(pool, "pool") if pool is not None else None
    fid = None
    if frame_ids is not None:
        if frame_ids.dtype != torch.int32 or not frame_ids.is_cuda or frame_ids.numel() < grid.T:
            raise ValueError("frame_ids must be a CUDA int32 tensor with one entry per logical frame")
        fid = frame_ids.contiguous().data_ptr()
    L.check(lib.li_tile_pool(L.ptr(v0), L.ptr(v1), fid, grid, L.ptr(d0), L.ptr(d1), int(dst_block_offset),
                             L.ptr(pv), int(pool_block_offset), L.stream_ptr(src0.device)), "li_tile_pool")


def pool_blocks(x: torch.Tensor, T: int, LH: int, LW: int, tile, frame_ids=None, normalized: bool = False,
                out: Optional[torch.Tensor] = None, block_offset: int = 0) -> torch.Tensor:
    """Per-block mean of a raster tensor ``[B,H,L,D]`` -> ``[B,H,Nblk,D]`` (no tiled copy) —
    ``li_pool_blocks``. ``normalized``: the rows are ``F.normalize``-d in the same launch
    (the 'cosine' selection input). ``out``/``block_offset``: write into rows
    ``block_offset..`` of an existing pool."""
    lib = L.load()
    nt, nh, nw = grid_blocks(T, LH, LW, tile)
    B, H, _, D = x.shape
    pool = torch.empty((B, H, nt * nh * nw, D), device=x.device, dtype=x.dtype) if out is None else out
    fid = None
    if frame_ids is not None:
        if frame_ids.dtype != torch.int32 or not frame_ids.is_cuda or frame_ids.numel() < T:
            raise ValueError("frame_ids must be a CUDA int32 tensor with one entry per logical frame")
        fid = frame_ids.contiguous().data_ptr()
    L.check(lib.li_pool_blocks(L.ptr(L.view4(x, "src")), fid, L.grid3d(T, LH, LW, tile), L.ptr(L.view4(pool, "pool")),
                               int(block_offset), 1 if normalized else 0, L.stream_ptr(x.device)), "li_pool_blocks")
    return pool


def pool_blocks_multi(jobs):
    """Several :func:`pool_blocks` jobs in one launch — ``li_pool_blocks_multi``. Each
    job is a dict with ``src``, ``T``, ``LH``, ``LW``, ``tile``, ``out`` (the pool
    tensor) and optionally ``block_offset``, ``normalized`` and ``frame_ids``; the
    pools are written in place (bit-identical to one ``pool_blocks`` call each)."""
    import ctypes
    lib = L.load()
    arr = (L.PoolJob * len(jobs))()
    keep = []
    for i, j in enumerate(jobs):
        sv, pv = L.view4(j["src"], "src"), L.view4(j["out"], "pool")
        keep += [sv, pv]
        arr[i].src, arr[i].pool = ctypes.pointer(sv), ctypes.pointer(pv)
        fid = j.get("frame_ids")
        if fid is not None:
            if fid.dtype != torch.int32 or not fid.is_cuda or not fid.is_contiguous() or fid.numel() < j["T"]:
                raise ValueError("frame_ids must be a contiguous CUDA int32 tensor with one entry per logical frame")
            arr[i].frame_ids = fid.data_ptr()
        arr[i].grid = L.grid3d(j["T"], j["LH"], j["LW"], j["tile"])
        arr[i].pool_block_offset = int(j.get("block_offset", 0))
        arr[i].normalized = 1 if j.get("normalized", False) else 0
    L.check(lib.li_pool_blocks_multi(arr, len(jobs), L.stream_ptr(jobs[0]["src"].device)), "li_pool_blocks_multi")


def text_blocks(k_txt, v_txt, bs: int, k_all, v_all):
    lib = L.load()
    L.check(lib.li_text_blocks(L.ptr(L.view4(k_txt, "k_txt")), L.ptr(L.view4(v_txt, "v_txt")), int(bs),
                               L.ptr(L.view5(k_all, "k_all")), L.ptr(L.view5(v_all, "v_all")),
                               L.stream_ptr(k_txt.device)), "li_text_blocks")


def untile(src: torch.Tensor, dst: torch.Tensor, grid: L.Grid3d):
    lib = L.load()
    L.check(lib.li_untile(L.ptr(L.view5(src, "src")), grid, L.ptr(L.view4(dst, "dst")),
                          L.stream_ptr(dst.device)), "li_untile")


def gather_frames(src: torch.Tensor, frame_ids: torch.Tensor, frame_tokens: int,
                  out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Retained-frame gather ``src[:, :, frames]`` on a ``[B,H,F*HW,D]`` pool — ``li_gather_frames``."""
    lib = L.load()
    if frame_ids.dtype != torch.int32 or not frame_ids.is_cuda:
        raise ValueError("frame_ids must be a CUDA int32 tensor")
    frame_ids = frame_ids.contiguous()
    n = frame_ids.numel()
    B, H, _, D = src.shape
    if out is None:
        out = torch.empty((B, H, n * frame_tokens, D), device=src.device, dtype=src.dtype)
    L.check(lib.li_gather_frames(L.ptr(L.view4(src, "src")), frame_ids.data_ptr(), int(n), int(frame_tokens),
                                 L.ptr(L.view4(out, "out")), error_word(src.device).data_ptr(),
                                 L.stream_ptr(src.device)), "li_gather_frames")
    return out


def metric_code(metric: str) -> int:
    if metric == "cosine":
        return L.METRIC_COSINE
    if metric == "scaled_dot_product":
        return L.METRIC_SCALED_DOT
    return L.METRIC_DOT


def select_params(mode: int, metric: str, tile, grid_q, grid_k, text_len: int, recent_protect: int = 0,
                  topk_ratio: float = 1.0, min_budget: int = 7, q_block_offset: int = 0) -> L.SelectParams:
    p = L.SelectParams()
    p.mode = mode
    p.metric = metric_code(metric)
    p.tt, p.th, p.tw = (int(x) for x in tile)
    for i in range(3):
        p.grid_q[i] = int(grid_q[i])
        p.grid_k[i] = int(grid_k[i])
    p.text_len = int(text_len)
    p.recent_protect = int(recent_protect)
    p.topk_ratio = float(topk_ratio)
    p.min_budget = int(min_budget)
    p.q_block_offset = int(q_block_offset)
    return p


def select_budget(p: L.SelectParams, nq: int, nk: int) -> Tuple[int, int]:
    import ctypes
    lib = L.load()
    ntxt, k = ctypes.c_int32(), ctypes.c_int32()
    L.check(lib.li_select_budget(ctypes.byref(p), int(nq), int(nk), ctypes.byref(ntxt), ctypes.byref(k)),
            "li_select_budget")
    return ntxt.value, k.value


def select_blocks(q_pool: torch.Tensor, k_pool: torch.Tensor, p: L.SelectParams,
                  score_bias: Optional[torch.Tensor] = None, return_rank: bool = False,
                  use_workspace: bool = True):
    """Block selection on pooled tensors — ``li_select_blocks``. Returns
    ``(indices, counts)`` (and the fp32 ranking scores with ``return_rank``).
    With ``use_workspace`` the scores and the top-k run as two wide kernels
    through a scratch buffer from torch's allocator; without it one kernel."""
    import ctypes
    lib = L.load()
    B, H, nq, _ = q_pool.shape
    nk = k_pool.shape[2]
    ntxt, k = select_budget(p, nq, nk)
    dev = q_pool.device
    idx = torch.empty((B, H, nq, ntxt + k), device=dev, dtype=torch.int32)
    cnt = torch.empty((B, H, nq), device=dev, dtype=torch.int32)
    rank = torch.empty((B, H, nq, nk), device=dev, dtype=torch.float32) if return_rank else None
    bias_v = None
    if score_bias is not None:
        score_bias = score_bias.to(torch.float32).expand(B, H, nq, nk)
        bias_v = L.view4(score_bias, "score_bias")
    ws, wsb = None, 0
    if use_workspace:
        nb = ctypes.c_int64()
        L.check(lib.li_select_workspace_bytes(B, H, nq, nk, ctypes.byref(nb)), "li_select_workspace_bytes")
        if nb.value:
            ws, wsb = torch.empty(nb.value, dtype=torch.uint8, device=dev), nb.value
    iv = L.index_view(idx, cnt)
    rv = L.view4(rank, "rank") if rank is not None else None
    L.check(lib.li_select_blocks(L.ptr(L.view4(q_pool, "q_pool")), L.ptr(L.view4(k_pool, "k_pool")), L.ptr(p),
                                 L.ptr(bias_v), L.ptr(iv), L.ptr(rv), ws.data_ptr() if ws is not None else None,
                                 int(wsb), L.stream_ptr(dev)), "li_select_blocks")
    return (idx, cnt, rank) if return_rank else (idx, cnt)


def normalize_rows(x: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``F.normalize(x, dim=-1)`` of pooled rows with the selection's rounding — ``li_normalize_rows``."""
    lib = L.load()
    y = torch.empty_like(x) if out is None else out
    L.check(lib.li_normalize_rows(L.ptr(L.view4(x, "x")), L.ptr(L.view4(y, "y")), L.stream_ptr(x.device)),
            "li_normalize_rows")
    return y


def rank_blocks(rank_scores: torch.Tensor, score_dtype: torch.dtype, k: int, text_len: int, bs: int):
    """Top-k + sort + text prepend on given ranking scores — ``li_rank_blocks``."""
    lib = L.load()
    rank_scores = rank_scores.to(torch.float32)
    B, H, nq, nk = rank_scores.shape
    ntxt = (text_len + bs - 1) // bs
    idx = torch.empty((B, H, nq, ntxt + k), device=rank_scores.device, dtype=torch.int32)
    cnt = torch.empty((B, H, nq), device=rank_scores.device, dtype=torch.int32)
    L.check(lib.li_rank_blocks(L.ptr(L.view4(rank_scores, "rank_scores")), L._DT[score_dtype], int(k),
                               int(text_len), int(bs), L.ptr(L.index_view(idx, cnt)),
                               L.stream_ptr(rank_scores.device)), "li_rank_blocks")
    return idx, cnt


def _attn_operand(t: torch.Tensor) -> torch.Tensor:
    """Attention operands: bf16/fp16 with D contiguous and 16-byte strides
    (copy only when the caller's layout cannot be described to TMA).

    fp32 operands become fp16: the reference's HY kernel feeds fp32 q/k/v to
    ``tl.dot`` (tf32: 10 explicit mantissa bits, ``longcat_kernel.py`` HY
    ``:126,141``), and fp16 keeps the same 10 bits, so the fp32 path computes at
    the reference's precision. A finite fp32 value beyond fp16's range (|x| >
    65504) would turn into an infinity: that sets ``LI_DEVERR_RANGE`` in the
    device error word (no host synchronisation), which
    :func:`raise_device_errors` reports."""
    if t.dtype == torch.float32:
        h = t.to(torch.float16)
        flag = (torch.isinf(h) & torch.isfinite(t)).any().to(torch.int32) * L.LI_DEVERR_RANGE
        error_word(t.device).bitwise_or_(flag)
        t = h
    elif t.dtype not in (torch.bfloat16, torch.float16):
        t = t.to(torch.bfloat16)
    ok = t.stride(-1) == 1 and all((s * 2) % 16 == 0 for s in t.stride()[:-1]) and t.data_ptr() % 16 == 0
    return t if ok else t.contiguous()


def attn_workspace(B: int, H: int, nq: int, smax: int, D: int, device, bs: int = 128):
    """Split-KV scratch for one attention call (``li_sparse_attn_workspace_bytes``),
    from torch's caching allocator; ``(tensor or None, bytes)``."""
    import ctypes
    lib = L.load()
    nbytes = ctypes.c_int64()
    L.check(lib.li_sparse_attn_workspace_bytes(int(B), int(H), int(nq), int(smax), int(D), int(bs),
                                               ctypes.byref(nbytes)), "li_sparse_attn_workspace_bytes")
    if nbytes.value == 0:
        return None, 0
    return torch.empty(nbytes.value, dtype=torch.uint8, device=device), nbytes.value


def sparse_attn_tiled(q, k, v, indices, counts, bs: int, sm_scale: Optional[float] = None,
                      return_lse: bool = False):
    """Block-sparse attention over tiled tensors — ``li_sparse_attn_tiled``."""
    lib = L.load()
    out_dtype = q.dtype
    q, k, v = _attn_operand(q), _attn_operand(k), _attn_operand(v)
    if k.dtype != q.dtype:
        k = k.to(q.dtype)
    if v.dtype != q.dtype:
        v = v.to(q.dtype)
    D = q.shape[-1]
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(D)
    o = torch.empty(q.shape, device=q.device, dtype=q.dtype)
    nq = (q.shape[2] + bs - 1) // bs
    lse = torch.empty((q.shape[0], q.shape[1], nq * bs), device=q.device, dtype=torch.float32) if return_lse else None
    ws, wsb = attn_workspace(q.shape[0], q.shape[1], nq, indices.shape[3], D, q.device, bs)
    L.check(lib.li_sparse_attn_tiled(L.ptr(L.view4(q, "q")), L.ptr(L.view4(k, "k")), L.ptr(L.view4(v, "v")),
                                     L.ptr(L.index_view(indices, counts)), int(bs), float(sm_scale),
                                     L.ptr(L.view4(o, "o")), lse.data_ptr() if lse is not None else None,
                                     error_word(q.device).data_ptr(), ws.data_ptr() if ws is not None else None,
                                     int(wsb), L.stream_ptr(q.device)),
            "li_sparse_attn_tiled")
    if o.dtype != out_dtype:
        o = o.to(out_dtype)
    return (o, lse) if return_lse else o


def sparse_attn_raster(q, grid_q: L.Grid3d, k_txt, v_txt, k_vis, v_vis, grid_k: L.Grid3d, indices, counts,
                       sm_scale: Optional[float] = None, return_lse: bool = False,
                       out: Optional[torch.Tensor] = None):
    """Fused tile -> block-sparse attention -> untile — ``li_sparse_attn_raster``."""
    lib = L.load()
    out_dtype = q.dtype
    q, k_vis, v_vis = _attn_operand(q), _attn_operand(k_vis), _attn_operand(v_vis)
    if k_vis.dtype != q.dtype:
        k_vis, v_vis = k_vis.to(q.dtype), v_vis.to(q.dtype)
    have_txt = k_txt is not None and k_txt.shape[2] > 0
    if have_txt:
        k_txt, v_txt = _attn_operand(k_txt).to(q.dtype), _attn_operand(v_txt).to(q.dtype)
    D = q.shape[-1]
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(D)
    if out is not None and out.dtype == q.dtype:
        o = out
    else:
        o = torch.empty(q.shape, device=q.device, dtype=q.dtype)
    bs = grid_q.tt * grid_q.th * grid_q.tw
    nt, nh, nw = grid_blocks(grid_q.T, grid_q.LH, grid_q.LW, (grid_q.tt, grid_q.th, grid_q.tw))
    lse = (torch.empty((q.shape[0], q.shape[1], nt * nh * nw * bs), device=q.device, dtype=torch.float32)
           if return_lse else None)
    ws, wsb = attn_workspace(q.shape[0], q.shape[1], nt * nh * nw, indices.shape[3], D, q.device, bs)
    L.check(lib.li_sparse_attn_raster(
        L.ptr(L.view4(q, "q")), grid_q, L.ptr(L.view4(k_txt, "k_txt")) if have_txt else None,
        L.ptr(L.view4(v_txt, "v_txt")) if have_txt else None, L.ptr(L.view4(k_vis, "k_vis")),
        L.ptr(L.view4(v_vis, "v_vis")), grid_k, L.ptr(L.index_view(indices, counts)), float(sm_scale),
        L.ptr(L.view4(o, "o")), lse.data_ptr() if lse is not None else None, error_word(q.device).data_ptr(),
        ws.data_ptr() if ws is not None else None, int(wsb), L.stream_ptr(q.device)), "li_sparse_attn_raster")
    if o.dtype != out_dtype:
        o = o.to(out_dtype)
        if out is not None:
            out.copy_(o)
            o = out
    return (o, lse) if return_lse else o
