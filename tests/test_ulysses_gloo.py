"""The sequence<->head all-to-all of the head-sharded step, on CPU gloo ranks.

Two processes exchange seeded tensors; every rank must end up with all tokens
of its own head group (seq -> head) and get its sequence slice back
(head -> seq). Also checks that a rank which never joins makes the others fail
with a timeout error instead of hanging.
"""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, result_q):
    import datetime
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
    try:
        from light_interaction_project_b200.ulysses import head_to_seq, seq_to_head
        N, B, S, H, D = 3, 2, 8, 4, 16
        g = torch.Generator().manual_seed(0)
        full = torch.randn(N, B, S, H, D, generator=g)
        s = S // world
        mine = full[:, :, rank * s:(rank + 1) * s]                  # [N, B, s, H, D]
        out = seq_to_head(mine, world)                              # [S, N, B, hl, D]
        hl = H // world
        expect = full[:, :, :, rank * hl:(rank + 1) * hl].permute(2, 0, 1, 3, 4)
        ok1 = torch.equal(out, expect)
        o = out[:, 0].permute(1, 2, 0, 3).contiguous()              # [B, hl, S, D]
        back = head_to_seq(o, world)                                # [B, s, H, D]
        ok2 = torch.equal(back, full[0, :, rank * s:(rank + 1) * s])
        result_q.put((rank, ok1, ok2))
    finally:
        dist.destroy_process_group()


def test_all_to_all_round_trip_two_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    res = sorted(q.get(timeout=5) for _ in range(2))
    assert all(p.exitcode == 0 for p in procs)
    assert res == [(0, True, True), (1, True, True)]


def _qkv_worker(rank, world, port, result_q):
    """The rank-major QKV projection lands in the layout seq_to_head produces
    (integer-valued inputs, so every product and sum is exact in fp32)."""
    import datetime
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
    try:
        from light_interaction_project_b200.ulysses import qkv_to_head, rank_major_qkv_weight, seq_to_head
        S, hidden, H, D = 8, 12, 4, 16
        g = torch.Generator().manual_seed(1)
        x = torch.randint(-3, 4, (S, hidden), generator=g).float()
        w = torch.randint(-3, 4, (hidden, 3 * H * D), generator=g).float()
        s = S // world
        mine = x[rank * s:(rank + 1) * s]
        got = qkv_to_head(mine, rank_major_qkv_weight(w, world, H, D), world, H, D)
        want = seq_to_head((mine @ w).view(1, s, 3, H, D).permute(2, 0, 1, 3, 4), world)
        result_q.put((rank, tuple(got.shape) == tuple(want.shape) and torch.equal(got, want)))
    finally:
        dist.destroy_process_group()


def test_rank_major_qkv_projection_two_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_qkv_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    res = sorted(q.get(timeout=5) for _ in range(2))
    assert all(p.exitcode == 0 for p in procs)
    assert res == [(0, True), (1, True)]


def _lonely(port, result_q):
    import datetime
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    try:
        dist.init_process_group("gloo", rank=0, world_size=2, timeout=datetime.timedelta(seconds=3))
        result_q.put("joined")
    except Exception as e:  # the peer never joins: rendezvous times out
        result_q.put(type(e).__name__)


def test_missing_rank_times_out_instead_of_hanging():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_lonely, args=(_free_port(), q))
    p.start()
    p.join(timeout=120)
    assert p.exitcode == 0
    assert q.get(timeout=5) != "joined"
