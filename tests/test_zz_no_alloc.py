"""li_select_blocks_static: the selection entry point whose scratch is a fixed
array in the library's global memory. Called through the C ABI and compared
with li_select_blocks (two-kernel path, workspace from torch) on two
consecutive calls; the over-size rejection is checked on the host.

Collected last so that it also runs after every other test in one process."""

import ctypes

import pytest
import torch

from light_interaction_project_b200 import _lib as L
from light_interaction_project_b200 import kernels as K

STATIC_BYTES = 8 << 20  # LI_SELECT_STATIC_SCRATCH_BYTES


def _outputs(B, H, nq, width, nk, device):
    idx = torch.full((B, H, nq, width), -7, device=device, dtype=torch.int32)
    cnt = torch.full((B, H, nq), -7, device=device, dtype=torch.int32)
    rank = torch.full((B, H, nq, nk), float("nan"), device=device, dtype=torch.float32)
    return idx, cnt, rank


def _call_static(lib, qp, kp, p, bias, idx, cnt, rank):
    bv = L.view4(bias, "score_bias") if bias is not None else None
    return lib.li_select_blocks_static(L.ptr(L.view4(qp, "q_pool")), L.ptr(L.view4(kp, "k_pool")), L.ptr(p),
                                       L.ptr(bv), L.ptr(L.index_view(idx, cnt)), L.ptr(L.view4(rank, "rank")),
                                       L.stream_ptr(qp.device))


def _call_workspace(lib, qp, kp, p, bias, idx, cnt, rank):
    B, H, nq, _ = qp.shape
    nk = kp.shape[2]
    nb = ctypes.c_int64()
    L.check(lib.li_select_workspace_bytes(B, H, nq, nk, ctypes.byref(nb)), "li_select_workspace_bytes")
    assert nb.value > 0
    ws = torch.empty(nb.value, dtype=torch.uint8, device=qp.device)
    bv = L.view4(bias, "score_bias") if bias is not None else None
    L.check(lib.li_select_blocks(L.ptr(L.view4(qp, "q_pool")), L.ptr(L.view4(kp, "k_pool")), L.ptr(p), L.ptr(bv),
                                 L.ptr(L.index_view(idx, cnt)), L.ptr(L.view4(rank, "rank")), ws.data_ptr(),
                                 nb.value, L.stream_ptr(qp.device)), "li_select_blocks")


CASES = [
    # (mode, metric, dtype, B, H, grid_q, grid_k, tile, text_len, recent_protect, ratio, bias)
    # batch*heads*Nq*Nk*4 = 1*32*64*1024*4 bytes: exactly the static buffer.
    (L.SELECT_DECODE, "scaled_dot_product", torch.bfloat16, 1, 32, (4, 4, 4), (64, 4, 4), (1, 8, 16), 0, 4, 0.25,
     True),
    (L.SELECT_DECODE, "dot", torch.bfloat16, 2, 3, (1, 8, 7), (16, 8, 7), (4, 4, 8), 77, 2, 0.3, False),
    (L.SELECT_BIDIR, "scaled_dot_product", torch.float16, 1, 4, (2, 4, 4), (2, 4, 4), (2, 4, 8), 300, 0, 0.3,
     False),
]


@pytest.mark.gpu
@pytest.mark.parametrize("case", CASES)
def test_static_scratch_matches_workspace_path(cuda_ok, case):
    mode, metric, dt, B, H, gq, gk, tile, text_len, rp, ratio, with_bias = case
    lib = L.load()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    nq, nk, D = gq[0] * gq[1] * gq[2], gk[0] * gk[1] * gk[2], 128
    p = K.select_params(mode, metric, tile, gq, gk, text_len, rp, ratio)
    ntxt, kb = K.select_budget(p, nq, nk)
    gen = torch.Generator(device=dev)
    for call in range(2):  # two consecutive calls on different inputs share the one scratch array
        gen.manual_seed(1000 + call)
        qp = (0.3 * torch.randn((B, H, nq, D), device=dev, generator=gen)).to(dt)
        kp = (0.3 * torch.randn((B, H, nk, D), device=dev, generator=gen)).to(dt)
        bias = torch.randn((B, H, nq, nk), device=dev, generator=gen).exp() if with_bias else None
        want = _outputs(B, H, nq, ntxt + kb, nk, dev)
        _call_workspace(lib, qp, kp, p, bias, *want)
        got = _outputs(B, H, nq, ntxt + kb, nk, dev)
        torch.cuda.synchronize()
        allocs_before = torch.cuda.memory_stats(dev).get("allocation.all.allocated", 0)
        free_before = torch.cuda.mem_get_info(dev)[0]
        L.check(_call_static(lib, qp, kp, p, bias, *got), "li_select_blocks_static")
        torch.cuda.synchronize()
        # No allocation through torch's allocator, and (a device-wide hint, since
        # another process could allocate meanwhile) no device memory reserved
        # after the first call's one-time address lookup.
        assert torch.cuda.memory_stats(dev).get("allocation.all.allocated", 0) == allocs_before
        if call:
            assert torch.cuda.mem_get_info(dev)[0] == free_before
        assert torch.equal(got[0], want[0]), f"indices differ on call {call}"
        assert torch.equal(got[1], want[1]), f"counts differ on call {call}"
        assert torch.equal(got[2], want[2]), f"ranking scores differ on call {call}"
        assert int(got[1].min()) >= ntxt


def test_static_scratch_rejects_oversize():
    """One head more than the buffer holds is refused on the host, before any
    device work (the data pointers here are never dereferenced)."""
    lib = L.load()
    B, H, nq, nk, D = 1, 33, 64, 1024, 128
    assert B * H * nq * nk * 4 > STATIC_BYTES

    def view(shape, dtype):
        v = L.View4()
        v.data = 1 << 20
        v.dtype = dtype
        st = 1
        for i in range(3, -1, -1):
            v.shape[i] = shape[i]
            v.stride[i] = st
            st *= shape[i]
        return v

    p = K.select_params(L.SELECT_DECODE, "scaled_dot_product", (1, 8, 16), (4, 4, 4), (64, 4, 4), 0, 4, 0.25)
    ntxt, kb = K.select_budget(p, nq, nk)
    iv = L.IndexView()
    iv.indices = 1 << 21
    iv.counts = 1 << 22
    for i, s in enumerate((H * nq * (ntxt + kb), nq * (ntxt + kb), ntxt + kb, 1)):
        iv.stride[i] = s
    for i, s in enumerate((H * nq, nq, 1)):
        iv.count_stride[i] = s
    for i, s in enumerate((B, H, nq, ntxt + kb)):
        iv.shape[i] = s
    qv, kv = view((B, H, nq, D), L.DTYPE_BF16), view((B, H, nk, D), L.DTYPE_BF16)
    st = lib.li_select_blocks_static(ctypes.byref(qv), ctypes.byref(kv), ctypes.byref(p), None, ctypes.byref(iv),
                                     None, None)
    assert st == L.LI_ERR_UNSUPPORTED
    msg = lib.li_last_error().decode()
    assert "static buffer holds 8388608" in msg and "needs 8650752" in msg
