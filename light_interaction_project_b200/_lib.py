"""ctypes binding of the li_b200 C ABI (``include/li_b200.h``).

Loads ``_lib/libli_b200.so`` (built in-tree by ``build_lib.py``) and wraps
torch tensors into the plain-pointer views the ABI takes. Every wrapper raises
on a non-zero status; there is no fallback path — without the library the
operators cannot run.
"""

from __future__ import annotations

import ctypes
import os
import threading
from ctypes import POINTER, Structure, c_char_p, c_double, c_float, c_int32, c_int64, c_uint32, c_uint64, c_void_p

import torch

_PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_PKG, "_lib", "libli_b200.so")

LI_OK = 0
LI_ERR_INVALID_ARG = 1
LI_ERR_SHAPE = 2
LI_ERR_STRIDE = 3
LI_ERR_ALIGNMENT = 4
LI_ERR_OUT_OF_BOUNDS = 5
LI_ERR_UNSUPPORTED = 6
LI_ERR_CUDA = 7
LI_ERR_TIMEOUT = 8

LI_DEVERR_BAD_INDEX = 1
LI_DEVERR_TIMEOUT = 2
LI_DEVERR_RANGE = 4

DTYPE_BF16, DTYPE_FP16, DTYPE_FP32 = 0, 1, 2
METRIC_COSINE, METRIC_SCALED_DOT, METRIC_DOT = 0, 1, 2
SELECT_DECODE, SELECT_BIDIR = 0, 1

_DT = {torch.bfloat16: DTYPE_BF16, torch.float16: DTYPE_FP16, torch.float32: DTYPE_FP32}


class View4(Structure):
    _fields_ = [("data", c_void_p), ("shape", c_int64 * 4), ("stride", c_int64 * 4), ("dtype", c_int32)]


class View5(Structure):
    _fields_ = [("data", c_void_p), ("shape", c_int64 * 5), ("stride", c_int64 * 5), ("dtype", c_int32)]


class IndexView(Structure):
    _fields_ = [("indices", c_void_p), ("shape", c_int64 * 4), ("stride", c_int64 * 4),
                ("counts", c_void_p), ("count_stride", c_int64 * 3)]


class Grid3d(Structure):
    _fields_ = [("T", c_int32), ("LH", c_int32), ("LW", c_int32), ("tt", c_int32), ("th", c_int32), ("tw", c_int32)]


class PoolJob(Structure):
    _fields_ = [("src", POINTER(View4)), ("frame_ids", c_void_p), ("grid", Grid3d), ("pool", POINTER(View4)),
                ("pool_block_offset", c_int64), ("normalized", c_int32)]


A2A_MAX_RANKS = 8
IPC_HANDLE_BYTES = 64


class A2ADesc(Structure):
    _fields_ = [("src", c_void_p), ("src_chunk_stride", c_int64), ("src_row_stride", c_int64),
                ("rows", c_int64), ("row_bytes", c_int64), ("dst", c_void_p * A2A_MAX_RANKS),
                ("dst_bytes", c_int64), ("dst_offset", c_int64), ("dst_row_stride", c_int64),
                ("flags", c_void_p * A2A_MAX_RANKS), ("my_flags", c_void_p), ("counter", c_void_p),
                ("err_word", c_void_p), ("epoch_word", c_void_p), ("epoch", c_uint32), ("world", c_int32), ("rank", c_int32),
                ("split_bytes", c_int64), ("dst2", c_void_p * A2A_MAX_RANKS), ("dst2_bytes", c_int64),
                ("dst2_offset", c_int64), ("dst2_row_stride", c_int64)]


class SelectParams(Structure):
    _fields_ = [("mode", c_int32), ("metric", c_int32), ("tt", c_int32), ("th", c_int32), ("tw", c_int32),
                ("grid_q", c_int32 * 3), ("grid_k", c_int32 * 3), ("text_len", c_int32),
                ("recent_protect", c_int32), ("topk_ratio", c_double), ("min_budget", c_int32),
                ("q_block_offset", c_int32)]


_lib = None
_lock = threading.Lock()

# Argument types of every exported entry point (also checked by the CPU tests).
SIGNATURES = {
    "li_version": ([], c_char_p),
    "li_last_error": ([], c_char_p),
    "li_kernel_launches": ([], c_uint64),
    "li_tile_pool": ([POINTER(View4), POINTER(View4), c_void_p, Grid3d, POINTER(View5), POINTER(View5), c_int64,
                      POINTER(View4), c_int64, c_void_p], c_int32),
    "li_pool_blocks": ([POINTER(View4), c_void_p, Grid3d, POINTER(View4), c_int64, c_int32, c_void_p], c_int32),
    "li_pool_blocks_multi": ([POINTER(PoolJob), c_int32, c_void_p], c_int32),
    "li_text_blocks": ([POINTER(View4), POINTER(View4), c_int32, POINTER(View5), POINTER(View5), c_void_p], c_int32),
    "li_untile": ([POINTER(View5), Grid3d, POINTER(View4), c_void_p], c_int32),
    "li_gather_frames": ([POINTER(View4), c_void_p, c_int32, c_int32, POINTER(View4), c_void_p, c_void_p], c_int32),
    "li_select_budget": ([POINTER(SelectParams), c_int64, c_int64, POINTER(c_int32), POINTER(c_int32)], c_int32),
    "li_select_blocks": ([POINTER(View4), POINTER(View4), POINTER(SelectParams), POINTER(View4), POINTER(IndexView),
                          POINTER(View4), c_void_p, c_int64, c_void_p], c_int32),
    "li_select_workspace_bytes": ([c_int64, c_int64, c_int64, c_int64, POINTER(c_int64)], c_int32),
    "li_select_blocks_static": ([POINTER(View4), POINTER(View4), POINTER(SelectParams), POINTER(View4),
                                 POINTER(IndexView), POINTER(View4), c_void_p], c_int32),
    "li_normalize_rows": ([POINTER(View4), POINTER(View4), c_void_p], c_int32),
    "li_rank_blocks": ([POINTER(View4), c_int32, c_int32, c_int32, c_int32, POINTER(IndexView), c_void_p], c_int32),
    "li_ipc_alloc": ([c_int64, POINTER(c_void_p), c_void_p], c_int32),
    "li_ipc_open": ([c_void_p, POINTER(c_void_p)], c_int32),
    "li_ipc_close": ([c_void_p], c_int32),
    "li_ipc_free": ([c_void_p], c_int32),
    "li_a2a_push": ([POINTER(A2ADesc), c_void_p], c_int32),
    "li_sparse_attn_workspace_bytes": ([c_int64, c_int64, c_int64, c_int64, c_int32, c_int32, POINTER(c_int64)],
                                       c_int32),
    "li_sparse_attn_tiled": ([POINTER(View4), POINTER(View4), POINTER(View4), POINTER(IndexView), c_int32, c_float,
                              POINTER(View4), c_void_p, c_void_p, c_void_p, c_int64, c_void_p], c_int32),
    "li_sparse_attn_raster": ([POINTER(View4), Grid3d, POINTER(View4), POINTER(View4), POINTER(View4),
                               POINTER(View4), Grid3d, POINTER(IndexView), c_float, POINTER(View4), c_void_p,
                               c_void_p, c_void_p, c_int64, c_void_p], c_int32),
}


def load(path: str = LIB_PATH):
    """Load (once) and return the ctypes library; raises if it is missing."""
    global _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(path):
                raise RuntimeError(
                    f"li_b200 native library not found at {path}; build it with "
                    "`python -m light_interaction_project_b200.build_lib` (no fallback path exists)")
            lib = ctypes.CDLL(path)
            for name, (args, res) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.argtypes = args
                fn.restype = res
            _lib = lib
    return _lib


def last_error() -> str:
    return load().li_last_error().decode()


def kernel_launches() -> int:
    """Kernels this process has launched through the library so far."""
    return int(load().li_kernel_launches())


def check(status: int, what: str):
    if status == LI_OK:
        return
    msg = last_error()
    if status in (LI_ERR_CUDA, LI_ERR_TIMEOUT):
        raise RuntimeError(f"{what}: {msg}")
    if status == LI_ERR_UNSUPPORTED:
        raise NotImplementedError(f"{what}: {msg}")
    raise ValueError(f"{what}: {msg}")


def dtype_code(t: torch.Tensor) -> int:
    try:
        return _DT[t.dtype]
    except KeyError:
        raise TypeError(f"unsupported dtype {t.dtype}") from None


def _require_cuda(t: torch.Tensor, name: str):
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor (this backend has no CPU path)")


def view4(t: torch.Tensor, name: str = "tensor") -> View4:
    _require_cuda(t, name)
    if t.dim() != 4:
        raise ValueError(f"{name} must be 4-D, got {tuple(t.shape)}")
    v = View4()
    v.data = t.data_ptr()
    for i in range(4):
        v.shape[i] = t.shape[i]
        v.stride[i] = t.stride(i)
    v.dtype = dtype_code(t)
    return v


def view5(t: torch.Tensor, name: str = "tensor") -> View5:
    _require_cuda(t, name)
    if t.dim() != 5:
        raise ValueError(f"{name} must be 5-D, got {tuple(t.shape)}")
    v = View5()
    v.data = t.data_ptr()
    for i in range(5):
        v.shape[i] = t.shape[i]
        v.stride[i] = t.stride(i)
    v.dtype = dtype_code(t)
    return v


def index_view(indices: torch.Tensor, counts: torch.Tensor) -> IndexView:
    _require_cuda(indices, "indices")
    if indices.dtype != torch.int32 or counts.dtype != torch.int32:
        raise TypeError("block indices and counts must be int32")
    if indices.dim() != 4 or counts.dim() != 3:
        raise ValueError("indices must be [B,H,Nq,S] and counts [B,H,Nq]")
    v = IndexView()
    v.indices = indices.data_ptr()
    for i in range(4):
        v.shape[i] = indices.shape[i]
        v.stride[i] = indices.stride(i)
    v.counts = counts.data_ptr()
    for i in range(3):
        v.count_stride[i] = counts.stride(i)
    return v


def grid3d(T, LH, LW, tile) -> Grid3d:
    g = Grid3d()
    g.T, g.LH, g.LW = int(T), int(LH), int(LW)
    g.tt, g.th, g.tw = (int(x) for x in tile)
    return g


def stream_ptr(device=None) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def ptr(t):
    return None if t is None else ctypes.byref(t)
