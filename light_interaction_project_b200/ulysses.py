"""Head-sharded multi-GPU step: Ulysses sequence<->head all-to-all around the
block-sparse attention.

The upstream attention processors shard the sequence across ranks and, before
attention, re-lay q/k/v from ``[B, S/P, H, D]`` to ``[B, S, H/P, D]`` with
``all_to_all_4D(x, scatter_dim=2, gather_dim=1)``; after attention the output
goes back with ``all_to_all_4D(o, scatter_dim=1, gather_dim=2)``
(hy-worldplay/patches/0001-integrate-acceleration.patch:646-654,744-745).
Selection and attention are independent per (b, h), so with heads split the
sparse op itself needs no communication.

Here the exchange is one all-to-all per direction over the q/k/v stack (one
exchange for all three), on the current stream: NCCL ``all_to_all_single``, or
``PeerExchange`` (``li_a2a_push``: 16-byte stores into the peers' CUDA-IPC
receive buffers). The attention reads q straight from the all-to-all output
through a strided view (no re-layout copy). With batch 1 each layer's resident
K/V is token-major, so the current chunk's K/V rows are one contiguous block at
its tail: the K/V projection writes them there directly at N = 1, and at N > 1
the peer exchange stores each token's k and v straight into the owning rank's
resident buffer (IPC-shared) while its q goes to the receive buffer. (The
reference concatenates the cached context with the new chunk on every call,
``hy patch:681-691``, which copies all of it.) A whole step can be captured as
one CUDA graph (:meth:`HeadShardedStack.capture`).
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import List, Optional

import torch
import torch.distributed as dist

from . import _lib as L
from . import bi_sparse_operation as mg
from . import kernels as K
from .memory import KeyPoolCache


def seq_to_head(x: torch.Tensor, world: int, group=None) -> torch.Tensor:
    """``[N, B, s, H, D]`` (N stacked tensors, s = S/P local tokens) ->
    ``[P*s, N, B, H/P, D]`` (all tokens, this rank's heads), contiguous."""
    N, B, s, H, D = x.shape
    if world == 1:
        return x.permute(2, 0, 1, 3, 4).contiguous()
    hl = H // world
    send = x.reshape(N, B, s, world, hl, D).permute(3, 2, 0, 1, 4, 5).contiguous()  # [P, s, N, B, hl, D]
    recv = torch.empty_like(send)
    dist.all_to_all_single(recv, send, group=group)
    return recv.reshape(world * s, N, B, hl, D)


def rank_major_qkv_weight(w_qkv: torch.Tensor, world: int, heads: int, head_dim: int) -> torch.Tensor:
    """``[hidden, 3*H*D]`` QKV weight (columns ``(q|k|v, head, d)``) -> ``[P, hidden, 3*(H/P)*D]``:
    block p holds the q/k/v columns of rank p's heads, so ``x @ w`` (batched over p) is
    already the all-to-all send buffer ``[P, s, 3, H/P, D]`` — no pack copy."""
    hidden = w_qkv.shape[0]
    hl = heads // world
    return (w_qkv.view(hidden, 3, world, hl, head_dim).permute(2, 0, 1, 3, 4)
            .reshape(world, hidden, 3 * hl * head_dim).contiguous())


def qkv_to_head(x2d: torch.Tensor, w_rank_major: torch.Tensor, world: int, heads: int, head_dim: int,
                group=None) -> torch.Tensor:
    """QKV projection of this rank's ``s`` tokens (batch 1) straight into the
    all-to-all send order, then the exchange: returns ``[P*s, 3, 1, H/P, D]``
    (all tokens, this rank's heads), the layout :func:`seq_to_head` returns."""
    s = x2d.shape[0]
    send = torch.matmul(x2d, w_rank_major)                 # [P, s, 3*hl*D]
    recv = torch.empty_like(send)
    dist.all_to_all_single(recv, send, group=group)
    return recv.view(world * s, 3, 1, heads // world, head_dim)


class _DeviceBuffer:
    """A raw device allocation seen by torch through ``__cuda_array_interface__``."""

    def __init__(self, ptr: int, nbytes: int, device_index: int):
        self.__cuda_array_interface__ = {"shape": (nbytes // 2,), "typestr": "<u2", "data": (ptr, False),
                                         "version": 3, "strides": None}
        self.device_index = device_index


class PeerExchange:
    """One all-to-all pattern over NVLink peer memory (``li_a2a_push``).

    Each rank allocates two receive buffers (alternating by call parity) and a
    flag array through CUDA IPC, exchanges the handles over the process group
    once, and maps its peers' buffers. A call pushes chunk p of the send buffer
    into rank p's receive buffer and returns, on the current stream, once this
    rank's receive buffer is complete. Every rank must make the same calls in the
    same order; one exchange serves one stream.

    A peer that does not arrive within 2 s makes the call set
    ``LI_DEVERR_TIMEOUT`` in the device error word and return. After that the
    exchange must not be used again (a late peer may still write into the
    receive buffers): :meth:`close` it and build a new one.
    """

    def __init__(self, recv_bytes: int, rank: int, world: int, device, group=None):
        import ctypes
        from . import _lib as L
        if world > L.A2A_MAX_RANKS:
            raise ValueError(f"peer exchange supports up to {L.A2A_MAX_RANKS} ranks")
        self.L, self.lib = L, L.load()
        self.rank, self.world, self.device, self.group = rank, world, torch.device(device), group
        self.recv_bytes = (int(recv_bytes) + 255) // 256 * 256
        self.own, self.mapped = [], []
        handles = []
        for nbytes in (self.recv_bytes, self.recv_bytes, 256):     # recv[0], recv[1], flags
            ptr, h = ctypes.c_void_p(), (ctypes.c_char * L.IPC_HANDLE_BYTES)()
            L.check(self.lib.li_ipc_alloc(nbytes, ctypes.byref(ptr), h), "li_ipc_alloc")
            self.own.append(ptr.value)
            handles.append(bytes(h))
        gathered = [None] * world
        dist.all_gather_object(gathered, handles, group=group)
        self.peers = []                                               # [rank][recv0, recv1, flags]
        for p in range(world):
            if p == rank:
                self.peers.append(list(self.own))
                continue
            ptrs = []
            for hb in gathered[p]:
                ptr = ctypes.c_void_p()
                L.check(self.lib.li_ipc_open(hb, ctypes.byref(ptr)), "li_ipc_open")
                self.mapped.append(ptr.value)
                ptrs.append(ptr.value)
            self.peers.append(ptrs)
        self.counter = torch.zeros(4, dtype=torch.int32, device=self.device)
        self.epoch = 0
        self.views = [torch.as_tensor(_DeviceBuffer(self.own[i], self.recv_bytes, self.device.index),
                                      device=self.device) for i in range(2)]
        dist.barrier(group=group)

    def recv_view(self, parity: int, dtype=torch.bfloat16) -> torch.Tensor:
        return self.views[parity].view(dtype)

    def push(self, src: torch.Tensor, rows: int, row_bytes: int, src_chunk_stride: int, src_row_stride: int,
             dst_offset: int, dst_row_stride: int, split=None) -> torch.Tensor:
        """Exchange; returns this rank's receive buffer (flat, dtype of ``src``).

        ``split`` = ``(split_bytes, dst2_ptrs, dst2_bytes, dst2_offset, dst2_row_stride)``:
        the first ``split_bytes`` of every row go to the receive buffers as above,
        the rest to ``dst2_ptrs[p]`` (one device pointer per rank, e.g. a
        :class:`SharedBuffers` allocation) at ``dst2_offset + r * dst2_row_stride``."""
        L = self.L
        if not src.is_cuda or src.device != self.device:
            raise ValueError("send buffer must be on this rank's device")
        span = (self.world - 1) * src_chunk_stride + (rows - 1) * src_row_stride + row_bytes
        if not src.is_contiguous() or span > src.numel() * src.element_size():
            raise ValueError("send buffer must be contiguous and cover the exchange pattern")
        self.epoch += 1
        parity = self.epoch & 1
        d = L.A2ADesc()
        d.src = src.data_ptr()
        d.src_chunk_stride, d.src_row_stride = src_chunk_stride, src_row_stride
        d.rows, d.row_bytes = rows, row_bytes
        for p in range(self.world):
            d.dst[p] = self.peers[p][parity]
            d.flags[p] = self.peers[p][2]
        d.dst_bytes, d.dst_offset, d.dst_row_stride = self.recv_bytes, dst_offset, dst_row_stride
        d.my_flags = self.own[2]
        d.counter = self.counter.data_ptr()
        d.err_word = K.error_word(self.device).data_ptr()
        # The epoch lives on the device (counter[1]); the host count only picks the
        # receive buffer, so a captured graph replays with fresh epochs.
        d.epoch_word = self.counter.data_ptr() + 4
        d.epoch, d.world, d.rank = self.epoch & 0xFFFFFFFF, self.world, self.rank
        if split is not None:
            d.split_bytes = split[0]
            for q in range(self.world):
                d.dst2[q] = split[1][q]
            d.dst2_bytes, d.dst2_offset, d.dst2_row_stride = split[2], split[3], split[4]
        L.check(self.lib.li_a2a_push(L.ptr(d), L.stream_ptr(self.device)), "li_a2a_push")
        return self.recv_view(parity, src.dtype)

    def close(self):
        """Unmaps the peers' buffers and frees this rank's (call after the last use
        has completed on every rank)."""
        for p in self.mapped:
            self.lib.li_ipc_close(p)
        for p in self.own:
            self.lib.li_ipc_free(p)
        self.mapped, self.own = [], []


class SharedBuffers:
    """Device buffers that every rank's peer exchange may write into: each rank
    allocates ``len(nbytes)`` zeroed buffers through CUDA IPC (``li_ipc_alloc``),
    the handles are exchanged once over the process group, and every rank maps
    its peers' buffers. ``tensor(i)`` is this rank's buffer ``i`` as a bf16
    tensor; ``ptrs(i)`` lists buffer ``i`` of every rank (a peer's as mapped here)."""

    def __init__(self, nbytes: List[int], rank: int, world: int, device, group=None):
        import ctypes
        self.L, self.lib = L, L.load()
        self.rank, self.world, self.device = rank, world, torch.device(device)
        self.nbytes = [int(n) for n in nbytes]
        self.own, self.mapped, handles = [], [], []
        for n in self.nbytes:
            ptr, h = ctypes.c_void_p(), (ctypes.c_char * L.IPC_HANDLE_BYTES)()
            L.check(self.lib.li_ipc_alloc(n, ctypes.byref(ptr), h), "li_ipc_alloc")
            self.own.append(ptr.value)
            handles.append(bytes(h))
        gathered = [None] * world
        dist.all_gather_object(gathered, handles, group=group)
        self._ptrs = [[0] * world for _ in self.nbytes]
        for p in range(world):
            for i, hb in enumerate(gathered[p]):
                if p == rank:
                    self._ptrs[i][p] = self.own[i]
                    continue
                ptr = ctypes.c_void_p()
                L.check(self.lib.li_ipc_open(hb, ctypes.byref(ptr)), "li_ipc_open")
                self.mapped.append(ptr.value)
                self._ptrs[i][p] = ptr.value
        self._views = [torch.as_tensor(_DeviceBuffer(self.own[i], n, self.device.index), device=self.device)
                       .view(torch.bfloat16) for i, n in enumerate(self.nbytes)]
        dist.barrier(group=group)

    def tensor(self, i: int) -> torch.Tensor:
        return self._views[i]

    def ptrs(self, i: int) -> List[int]:
        return self._ptrs[i]

    def close(self):
        """Unmaps the peers' buffers and frees this rank's (after the last use has
        completed on every rank)."""
        self._views = []
        for p in self.mapped:
            self.lib.li_ipc_close(p)
        for p in self.own:
            self.lib.li_ipc_free(p)
        self.mapped, self.own = [], []


def head_to_seq(o: torch.Tensor, world: int, group=None) -> torch.Tensor:
    """``[B, H/P, S, D]`` (this rank's heads, all tokens) -> ``[B, S/P, H, D]``."""
    B, hl, S, D = o.shape
    if world == 1:
        return o.permute(0, 2, 1, 3)
    s = S // world
    send = o.permute(2, 0, 1, 3).reshape(world, s, B, hl, D).contiguous()  # [P, s, B, hl, D]
    recv = torch.empty_like(send)
    dist.all_to_all_single(recv, send, group=group)
    return recv.permute(2, 1, 0, 3, 4).reshape(B, s, world * hl, D)


@dataclass
class StackConfig:
    layers: int = 30
    heads: int = 24
    head_dim: int = 128
    hidden: int = 3072
    latent_hw: tuple = (30, 52)
    query_frames: int = 4
    memory_frames: int = 64
    tile: tuple = (4, 4, 8)
    keep_ratio: float = 0.25
    metric: str = "cosine"
    batch: int = 1
    # N > 1: "nccl" (all_to_all_single) or "peer" (li_a2a_push over NVLink peer memory,
    # bit-identical; with the step captured as one CUDA graph the faster of the two:
    # 15.84 vs 16.06 ms per 30-layer step at 8 GPUs). The library default stays NCCL,
    # which needs no CUDA-IPC mappings; bench.py selects "peer" only after checking
    # it bit for bit against NCCL on the same box (its "exchange_check").
    exchange: str = "nccl"

    @property
    def frame_tokens(self):
        return self.latent_hw[0] * self.latent_hw[1]

    @property
    def q_tokens(self):
        return self.query_frames * self.frame_tokens

    @property
    def kv_frames(self):
        return self.memory_frames + self.query_frames

    def blocks(self):
        LH, LW = self.latent_hw
        nq = K.grid_blocks(self.query_frames, LH, LW, self.tile)
        nk = K.grid_blocks(self.kv_frames, LH, LW, self.tile)
        return nq[0] * nq[1] * nq[2], nk[0] * nk[1] * nk[2]

    def budget(self):
        _, nk = self.blocks()
        return min(max(int(nk * self.keep_ratio), 7), nk)

    def attention_flops(self, heads: Optional[int] = None) -> float:
        """Executed FLOPs of one attention call over the padded tiled layout."""
        nq, _ = self.blocks()
        bs = self.tile[0] * self.tile[1] * self.tile[2]
        h = self.heads if heads is None else heads
        return 4.0 * self.batch * h * nq * bs * self.budget() * bs * self.head_dim


class HeadShardedStack:
    """``layers`` attention layers of one query chunk, heads split over ``world``
    ranks: QKV projection -> all-to-all -> block-sparse attention over the
    resident (memory + current chunk) K/V -> all-to-all -> O projection."""

    def __init__(self, cfg: StackConfig, rank: int, world: int, device, group=None, seed: int = 0):
        if cfg.heads % world or cfg.q_tokens % world:
            raise ValueError("heads and query tokens must divide by the world size")
        self.cfg, self.rank, self.world, self.group = cfg, rank, world, group
        self.device = torch.device(device)
        self.hl = cfg.heads // world
        g = torch.Generator(device=self.device)
        g.manual_seed(seed + 1000 * rank)
        std = 1.0 / math.sqrt(cfg.hidden)
        dt = torch.bfloat16
        hd = cfg.heads * cfg.head_dim
        # Same weights on every rank (seeded without the rank).
        gw = torch.Generator(device=self.device)
        gw.manual_seed(seed)
        self.w_qkv = [(torch.randn(cfg.hidden, 3 * hd, generator=gw, device=self.device) * std).to(dt)
                      for _ in range(cfg.layers)]
        self.w_o = [(torch.randn(hd, cfg.hidden, generator=gw, device=self.device) * std).to(dt)
                    for _ in range(cfg.layers)]
        # Batch 1 keeps each layer's resident K/V token-major, [L, 2, H/P, D]: the current
        # chunk's K and V rows are then one contiguous [S, 2*(H/P)*D] block at the tail,
        # which the K/V projection (N = 1) or the peer exchange (N > 1) writes in place.
        # Larger batches keep [B, 2, H/P, L, D] and write the tail with one gather launch.
        self.token_major = cfg.batch == 1
        # N = 1, batch 1: the Q and the K/V projections are separate GEMMs, the second
        # writing straight into the resident buffer's tail.
        self.w_q = self.w_kv = None
        if world == 1 and self.token_major:
            self.w_q = [w[:, :hd].contiguous() for w in self.w_qkv]
            self.w_kv = [w[:, hd:].contiguous() for w in self.w_qkv]
        # N > 1, batch 1: the QKV projection writes the all-to-all send buffer directly.
        self.w_qkv_rank = ([rank_major_qkv_weight(w, world, cfg.heads, cfg.head_dim) for w in self.w_qkv]
                           if world > 1 and cfg.batch == 1 else None)
        kv_tokens = cfg.kv_frames * cfg.frame_tokens
        es = 2
        # N > 1, batch 1: both exchanges over NVLink peer memory. The input side sends
        # each token's q to the receive buffer and its k, v into the resident K/V
        # buffer of the rank that owns those heads (IPC-shared); the output side lands
        # directly in the [s, H, D] rows the O projection reads.
        self.ex_qkv = self.ex_out = self.kv_shared = None
        if world > 1 and cfg.batch == 1 and cfg.exchange == "peer":
            s = cfg.q_tokens // world
            self.ex_qkv = PeerExchange(world * s * self.hl * cfg.head_dim * es, rank, world, self.device, group)
            self.ex_out = PeerExchange(s * cfg.heads * cfg.head_dim * es, rank, world, self.device, group)
            self.kv_shared = SharedBuffers([kv_tokens * 2 * self.hl * cfg.head_dim * es] * cfg.layers, rank, world,
                                           self.device, group)
        self.kv_buf: List[torch.Tensor] = []
        self.k_buf: List[torch.Tensor] = []
        self.v_buf: List[torch.Tensor] = []
        for i in range(cfg.layers):
            if self.token_major:
                shape = (kv_tokens, 2, self.hl, cfg.head_dim)
                kv = (self.kv_shared.tensor(i).view(shape) if self.kv_shared is not None
                      else torch.empty(shape, device=self.device, dtype=dt))
                kv.copy_(torch.randn(shape, generator=g, device=self.device))
                self.kv_buf.append(kv)
                self.k_buf.append(kv[:, 0].permute(1, 0, 2).unsqueeze(0))    # [1, H/P, L, D] views
                self.v_buf.append(kv[:, 1].permute(1, 0, 2).unsqueeze(0))
            else:
                kv = torch.randn(cfg.batch, 2, self.hl, kv_tokens, cfg.head_dim, generator=g,
                                 device=self.device).to(dt)
                self.kv_buf.append(kv)
                self.k_buf.append(kv[:, 0])
                self.v_buf.append(kv[:, 1])
        nq, nk = cfg.blocks()
        self.q_block_offset = nk - nq
        # Batch > 1: identity frame list; the current chunk's K/V go into the buffer
        # tail through the library's 16-byte row-gather kernel.
        self.chunk_frames = torch.arange(cfg.query_frames, dtype=torch.int32, device=self.device)
        # Pooled keys per layer: the memory frames are pooled once, each step
        # re-pools only the current chunk's block rows.
        self.key_pools = [KeyPoolCache(cfg.latent_hw, cfg.tile, cfg.metric) for _ in range(cfg.layers)]
        self.params = {"tile_size": tuple(cfg.tile), "topk_ratio": cfg.keep_ratio, "sim_metric": cfg.metric}
        self._graph = None
        self.graph_launches = 0

    def local_tokens(self):
        return self.cfg.q_tokens // self.world

    def make_input(self, seed: int = 7) -> torch.Tensor:
        g = torch.Generator(device=self.device)
        g.manual_seed(seed + self.rank)
        return torch.randn(self.cfg.batch, self.local_tokens(), self.cfg.hidden, generator=g,
                           device=self.device).to(torch.bfloat16)

    def qkv_exchange(self, i: int, x: torch.Tensor) -> torch.Tensor:
        """Layer ``i``'s QKV projection and sequence->head exchange: writes the current
        chunk's K/V rows into the layer's resident buffer (all of its S tokens, this
        rank's heads) and returns q ``[B, H/P, S, D]`` (a strided view)."""
        cfg = self.cfg
        B, s, _ = x.shape
        D, hl = cfg.head_dim, self.hl
        S = s * self.world
        tail = self.k_buf[i].shape[2] - S
        if self.token_major and self.world == 1:
            # Q projection, and the K/V projection written straight into the tail rows.
            torch.matmul(x.reshape(s, cfg.hidden), self.w_kv[i], out=self.kv_buf[i][tail:].view(S, 2 * hl * D))
            return (x.reshape(s, cfg.hidden) @ self.w_q[i]).view(1, S, hl, D).permute(0, 2, 1, 3)
        if self.ex_qkv is not None:
            # One push per token row: q to the receive buffer, k and v straight into
            # the tail of the owning rank's resident K/V buffer.
            send = torch.matmul(x.reshape(B * s, cfg.hidden), self.w_qkv_rank[i])   # [P, s, 3*hl*D]
            row = 3 * hl * D * send.element_size()
            qb = hl * D * send.element_size()
            recv = self.ex_qkv.push(send, s, row, s * row, row, self.rank * s * qb, qb,
                                    split=(qb, self.kv_shared.ptrs(i), self.kv_shared.nbytes[i],
                                           (tail + self.rank * s) * 2 * qb, 2 * qb))
            return recv[: S * hl * D].view(1, S, hl, D).permute(0, 2, 1, 3)
        if self.w_qkv_rank is not None:
            full = qkv_to_head(x.reshape(B * s, cfg.hidden), self.w_qkv_rank[i], self.world, cfg.heads,
                               cfg.head_dim, self.group)                         # [S, 3, B, hl, D]
        else:
            qkv = (x.reshape(B * s, cfg.hidden) @ self.w_qkv[i]).view(B, s, 3, cfg.heads, cfg.head_dim)
            full = seq_to_head(qkv.permute(2, 0, 1, 3, 4), self.world, self.group)   # [S, 3, B, hl, D]
        if self.token_major:
            self.kv_buf[i][tail:].copy_(full[:, 1:3, 0])
        else:
            ft = cfg.frame_tokens
            K.gather_frames(full[:, 1].permute(1, 2, 0, 3), self.chunk_frames, ft, out=self.k_buf[i][:, :, tail:])
            K.gather_frames(full[:, 2].permute(1, 2, 0, 3), self.chunk_frames, ft, out=self.v_buf[i][:, :, tail:])
        return full[:, 0].permute(1, 2, 0, 3)                                    # [B, hl, S, D] view

    def layer(self, i: int, x: torch.Tensor, attn_events=None, marks=None) -> torch.Tensor:
        """Layer ``i``. ``marks`` (optional list): a timing event is recorded on the
        current stream before the layer and after each of its phases and appended as
        ``(phase, event)``: qkv_projection_and_exchange, pooling,
        selection_and_attention, output_exchange, o_projection."""
        def mark(name):
            if marks is not None:
                ev = torch.cuda.Event(enable_timing=True)
                ev.record()
                marks.append((name, ev))
        cfg = self.cfg
        B, s, _ = x.shape
        S = s * self.world
        mark("start")
        q = self.qkv_exchange(i, x)
        mark("qkv_projection_and_exchange")
        # The attention writes its output token-major ([B, S, H/P, D]), the order the
        # return all-to-all / O projection reads, so no re-layout copy follows.
        o_tok = torch.empty(B, S, self.hl, cfg.head_dim, device=x.device, dtype=x.dtype)
        # One pooling launch for q and the current chunk's rows of the cached key
        # pool (the memory frames' rows were pooled once and stay valid).
        LH, LW = cfg.latent_hw
        nq, _ = cfg.blocks()
        q_pool = torch.empty(B, self.hl, nq, cfg.head_dim, device=x.device, dtype=x.dtype)
        jobs = [dict(src=q, T=cfg.query_frames, LH=LH, LW=LW, tile=tuple(cfg.tile), out=q_pool,
                     normalized=cfg.metric == "cosine")]
        kjob = self.key_pools[i].pool_job(self.k_buf[i], changed_from_frame=cfg.memory_frames)
        if kjob is not None:
            jobs.append(kjob)
        K.pool_blocks_multi(jobs)
        mark("pooling")
        if attn_events is not None:
            attn_events[0].record()
        o = mg.run_sparse_attention(q, self.k_buf[i], self.v_buf[i], 0, i, cfg.latent_hw, self.params,
                                    q_block_offset=self.q_block_offset, out=o_tok.permute(0, 2, 1, 3),
                                    k_pool=self.key_pools[i], q_pool=q_pool)
        if attn_events is not None:
            attn_events[1].record()
        mark("selection_and_attention")
        if self.ex_out is not None:
            row = self.hl * cfg.head_dim * o_tok.element_size()
            recv = self.ex_out.push(o_tok, s, row, s * row, row, self.rank * row, cfg.heads * row // self.hl)
            back = recv[: s * cfg.heads * cfg.head_dim].view(B, s, cfg.heads, cfg.head_dim)
        else:
            back = head_to_seq(o, self.world, self.group)                       # [B, s, H, D]
        mark("output_exchange")
        # O projection with the residual add in the GEMM epilogue.
        y = torch.addmm(x.reshape(B * s, cfg.hidden), back.reshape(B * s, cfg.heads * cfg.head_dim),
                        self.w_o[i]).view(B, s, cfg.hidden)
        mark("o_projection")
        return y

    def close(self):
        """Releases the captured graph and the peer-exchange buffers (after the last
        step has completed on every rank). With the peer exchange the resident K/V
        buffers are IPC-shared memory freed here, so the stack has no layers left to
        run afterwards (build a new one)."""
        self._graph = None
        if self.kv_shared is not None:
            self.kv_buf, self.k_buf, self.v_buf = [], [], []
        for ex in (self.ex_qkv, self.ex_out, self.kv_shared):
            if ex is not None:
                ex.close()
        self.ex_qkv = self.ex_out = self.kv_shared = None

    def step(self, x: torch.Tensor, attn_events=None, check_errors: bool = False, marks=None) -> torch.Tensor:
        """One step of every layer. ``check_errors``: synchronise afterwards and raise if
        a kernel reported a device-side error (a bad block id, a bounded wait that
        gave up); device errors are otherwise only visible through
        ``kernels.raise_device_errors``. ``marks``: per-phase timing events of every
        layer (see :meth:`layer`)."""
        for i in range(self.cfg.layers):
            x = self.layer(i, x, attn_events[i] if attn_events is not None else None, marks)
        if check_errors:
            K.raise_device_errors(self.device)
        return x

    def capture(self, x: torch.Tensor, warmup: int = 2) -> torch.Tensor:
        """Records one :meth:`step` on the static input ``x`` into a CUDA graph and
        returns its static output; :meth:`replay` then runs the whole step (every
        kernel and exchange of every layer) as one graph launch. Refill ``x`` in
        place between replays. The warm-up steps run first on a side stream, so
        the key pools, workspaces and communicators exist before capture.

        Every rank captures the same steps. The peer exchanges keep their epoch on
        the device, and each alternates its two receive buffers by call parity, so
        a graph must contain an even number of calls per exchange (one per layer:
        an even layer count)."""
        dev = self.device
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            for _ in range(warmup):
                self.step(x)
        torch.cuda.current_stream(dev).wait_stream(side)
        exchanges = [ex for ex in (self.ex_qkv, self.ex_out) if ex is not None]
        before = [ex.epoch for ex in exchanges]
        graph = torch.cuda.CUDAGraph()
        n0 = L.kernel_launches()
        with torch.cuda.graph(graph):
            y = self.step(x)
        # library kernels one replay launches
        self.graph_launches = L.kernel_launches() - n0
        if any((ex.epoch - e0) % 2 for ex, e0 in zip(exchanges, before)):
            # Nothing captured has run: put the call counts back so the executed
            # calls keep alternating their receive buffers.
            for ex, e0 in zip(exchanges, before):
                ex.epoch = e0
            raise ValueError("a captured step must make an even number of calls per peer exchange")
        self._graph = (graph, y)
        return y

    def replay(self, check_errors: bool = False) -> torch.Tensor:
        """Runs the captured step on the current contents of its static input
        (``check_errors`` as in :meth:`step`)."""
        if self._graph is None:
            raise RuntimeError("HeadShardedStack.capture() has not been called")
        self._graph[0].replay()
        if check_errors:
            K.raise_device_errors(self.device)
        return self._graph[1]

    def release_graph(self):
        """Drops the captured graph (before the process group is destroyed)."""
        self._graph = None
