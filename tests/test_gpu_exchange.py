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
