"""Peer exchange (li_a2a_push over NVLink) on two GPUs: a head-sharded stack
step gives bit-identical outputs through the peer exchange and through NCCL,
eagerly and replayed from a captured CUDA graph.
Needs two GPUs (skipped otherwise); each rank is its own process."""

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank(rank, world, port, q):
    import datetime
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        from light_interaction_project_b200 import kernels as K
        from light_interaction_project_b200.ulysses import HeadShardedStack, StackConfig
        outs = {}
        for mode in ("peer", "nccl"):
            cfg = StackConfig(layers=2, heads=4, hidden=512, memory_frames=4, exchange=mode)
            st = HeadShardedStack(cfg, rank, world, dev, group=dist.group.WORLD)
            x = st.make_input()
            ys = [st.step(x) for _ in range(2)]       # two steps: both buffer parities, rising epochs
            # The same step as a captured CUDA graph (device-held epochs), replayed twice.
            xs = x.clone()
            yg = st.capture(xs)
            for _ in range(2):
                st.replay()
                torch.cuda.synchronize()
                ys.append(yg.clone())
            torch.cuda.synchronize()
            dist.barrier()
            st.close()
            outs[mode] = ys
        errs = K.device_errors(dev)
        same = all(torch.equal(a, b) for a, b in zip(outs["peer"], outs["nccl"]))
        same = same and all(torch.equal(outs[m][0], y) for m in outs for y in outs[m][1:])
        q.put((rank, same, int(errs)))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_peer_exchange_matches_nccl_two_gpus():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    assert all(p.exitcode == 0 for p in procs)
    res = sorted(q.get(timeout=5) for _ in range(2))
    assert res == [(0, True, 0), (1, True, 0)]


def _desc(L, K, src, dsts, flags, counter, rows, row_bytes, world, rank, dev):
    d = L.A2ADesc()
    d.src = src.data_ptr()
    d.src_chunk_stride, d.src_row_stride = rows * row_bytes, row_bytes
    d.rows, d.row_bytes = rows, row_bytes
    for p in range(world):
        d.dst[p] = dsts[p].data_ptr()
        d.flags[p] = flags[p].data_ptr()
    d.dst_bytes = dsts[0].numel() * dsts[0].element_size()
    d.dst_offset, d.dst_row_stride = 0, row_bytes
    d.my_flags = flags[rank].data_ptr()
    d.counter = counter.data_ptr()
    d.err_word = K.error_word(dev).data_ptr()
    d.epoch_word = counter.data_ptr() + 4
    d.epoch, d.world, d.rank = 0, world, rank
    return d


@pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a GPU")
def test_exchange_single_rank_completes():
    """world = 1: the push copies the one chunk into this rank's buffer and its own
    flag completes the barrier at once; the device epoch advances per call."""
    from light_interaction_project_b200 import _lib as L
    from light_interaction_project_b200 import kernels as K
    dev = torch.device("cuda", 0)
    K.device_errors(dev)
    rows, row_bytes = 37, 96
    src = torch.randint(0, 255, (rows * row_bytes,), dtype=torch.uint8, device=dev)
    dst = torch.zeros_like(src)
    flags = torch.zeros(4, dtype=torch.int32, device=dev)
    counter = torch.zeros(4, dtype=torch.int32, device=dev)
    lib = L.load()
    for call in range(1, 4):
        d = _desc(L, K, src, [dst], [flags], counter, rows, row_bytes, 1, 0, dev)
        L.check(lib.li_a2a_push(L.ptr(d), L.stream_ptr(dev)), "li_a2a_push")
        torch.cuda.synchronize()
        assert counter[1].item() == call and flags[0].item() == call and counter[0].item() == 0
    assert torch.equal(dst, src)
    assert K.device_errors(dev) == 0


@pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a GPU")
def test_exchange_split_rows_single_rank():
    """Split rows: the first split_bytes of every row land in the receive buffer, the
    rest in the second destination at its own offset and row stride (the stack
    sends q to the receive buffer and k, v into the resident K/V buffer's tail)."""
    from light_interaction_project_b200 import _lib as L
    from light_interaction_project_b200 import kernels as K
    dev = torch.device("cuda", 0)
    K.device_errors(dev)
    rows, row_bytes, split = 40, 96, 32
    src = torch.randint(0, 255, (rows, row_bytes), dtype=torch.uint8, device=dev)
    dst = torch.zeros(rows * split, dtype=torch.uint8, device=dev)
    dst2 = torch.zeros(8 * 128 + rows * 128, dtype=torch.uint8, device=dev)   # 8 rows of head room, stride 128
    flags = torch.zeros(4, dtype=torch.int32, device=dev)
    counter = torch.zeros(4, dtype=torch.int32, device=dev)
    d = _desc(L, K, src, [dst], [flags], counter, rows, row_bytes, 1, 0, dev)
    d.dst_row_stride = split
    d.split_bytes = split
    d.dst2[0] = dst2.data_ptr()
    d.dst2_bytes, d.dst2_offset, d.dst2_row_stride = dst2.numel(), 8 * 128, 128
    L.check(L.load().li_a2a_push(L.ptr(d), L.stream_ptr(dev)), "li_a2a_push")
    torch.cuda.synchronize()
    assert torch.equal(dst.view(rows, split), src[:, :split])
    body = dst2[8 * 128:].view(rows, 128)
    assert torch.equal(body[:, : row_bytes - split], src[:, split:])
    assert int(body[:, row_bytes - split:].abs().sum()) == 0 and int(dst2[: 8 * 128].abs().sum()) == 0
    assert K.device_errors(dev) == 0
    # A second destination too small for the rows is refused before any launch.
    d.dst2_bytes = 8 * 128 + (rows - 1) * 128 + 32
    assert L.load().li_a2a_push(L.ptr(d), L.stream_ptr(dev)) == L.LI_ERR_OUT_OF_BOUNDS


@pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a GPU")
def test_exchange_wait_runs_out_and_reports():
    """A peer that never joins: rank 0 of a world of 2 on one GPU, with nothing
    playing rank 1. The push still delivers both chunks (both buffers are local),
    raises its flags, and its bounded wait for rank 1's flag gives up after 2 s:
    LI_DEVERR_TIMEOUT in the error word, the epoch advanced, the context usable."""
    import time
    from light_interaction_project_b200 import _lib as L
    from light_interaction_project_b200 import kernels as K
    dev = torch.device("cuda", 0)
    K.device_errors(dev)
    rows, row_bytes = 64, 256
    src = torch.randint(0, 255, (2 * rows * row_bytes,), dtype=torch.uint8, device=dev)
    dsts = [torch.zeros(rows * row_bytes, dtype=torch.uint8, device=dev) for _ in range(2)]
    flags = [torch.zeros(4, dtype=torch.int32, device=dev) for _ in range(2)]
    counter = torch.zeros(4, dtype=torch.int32, device=dev)
    d = _desc(L, K, src, dsts, flags, counter, rows, row_bytes, 2, 0, dev)
    t0 = time.perf_counter()
    L.check(L.load().li_a2a_push(L.ptr(d), L.stream_ptr(dev)), "li_a2a_push")
    torch.cuda.synchronize()
    waited = time.perf_counter() - t0
    assert 1.5 < waited < 30.0
    assert K.device_errors(dev) & L.LI_DEVERR_TIMEOUT
    assert torch.equal(dsts[0], src[: rows * row_bytes]) and torch.equal(dsts[1], src[rows * row_bytes:])
    assert flags[0][0].item() == 1 and flags[1][0].item() == 1 and flags[0][1].item() == 0
    assert counter[1].item() == 1 and counter[0].item() == 0
    # the context is still usable
    x = torch.arange(1000, device=dev, dtype=torch.float32)
    assert float((x * 2).sum().item()) == 999000.0
