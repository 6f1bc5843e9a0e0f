"""GPU parity: tiling, block-mean pooling, frame gather, text blocks, untiling.

All integer/layout work is compared bit for bit with the oracle; the block
means follow the oracle's fixed fp64 summation order, so they too must match
bit for bit.
"""

import numpy as np
import pytest
import torch

from gpu_util import TORCH_DT, dev, rand, to_gpu, to_np
from light_interaction_project_b200 import _lib as L
from light_interaction_project_b200 import ar_sparse_operation as ar
from light_interaction_project_b200 import kernels as K
from light_interaction_project_b200 import memory
from oracle import li_oracle as O

pytestmark = pytest.mark.gpu

GEOMS = [
    # (B, H, D, T, LH, LW, tile)
    (1, 2, 128, 3, 30, 52, (1, 8, 16)),   # HY latent, partial blocks in h and w
    (1, 3, 128, 6, 30, 52, (4, 4, 8)),    # MG tile, partial t block (6 = 4 + 2)
    (2, 2, 128, 5, 12, 20, (4, 8, 4)),    # HY default tile
    (1, 4, 64, 6, 8, 8, (2, 4, 8)),       # toy config tile (64-token blocks)
]


@pytest.mark.parametrize("geom", GEOMS)
@pytest.mark.parametrize("dtype", ["bf16", "fp16", "fp32"])
def test_tile_pool_bit_exact(cuda_ok, geom, dtype):
    B, H, D, T, LH, LW, tile = geom
    x, tx = rand((B, H, T * LH * LW, D), 1000 + T, dtype)
    y, ty = rand((B, H, T * LH * LW, D), 2000 + T, dtype)
    nt, nh, nw = K.grid_blocks(T, LH, LW, tile)
    nblk = nt * nh * nw
    bs = tile[0] * tile[1] * tile[2]
    ntxt = 2
    kd = torch.full((B, H, ntxt + nblk, bs, D), float("nan"), device=dev(), dtype=TORCH_DT[dtype])
    vd = torch.full_like(kd, float("nan"))
    pool = torch.full((B, H, nblk, D), float("nan"), device=dev(), dtype=TORCH_DT[dtype])
    ar.launch_kv_prep(tx, ty, kd, vd, pool, ntxt, 0, T, LH, LW, *tile, nh, nw)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(to_np(kd[:, :, ntxt:]), O.tile_raster(x, T, LH, LW, tile))
    np.testing.assert_array_equal(to_np(vd[:, :, ntxt:]), O.tile_raster(y, T, LH, LW, tile))
    assert torch.isnan(kd[:, :, :ntxt].float()).all(), "text blocks must be left for li_text_blocks"
    np.testing.assert_array_equal(to_np(pool), O.block_mean(O.tile_raster(x, T, LH, LW, tile), dtype))


@pytest.mark.parametrize("dtype", ["bf16", "fp32"])
def test_q_prep_and_untile_round_trip(cuda_ok, dtype):
    B, H, D, T, LH, LW, tile = 2, 3, 128, 4, 30, 52, (1, 8, 16)
    x, tx = rand((B, H, T * LH * LW, D), 77, dtype)
    nt, nh, nw = K.grid_blocks(T, LH, LW, tile)
    bs = tile[0] * tile[1] * tile[2]
    qt = torch.empty((B, H, nt * nh * nw, bs, D), device=dev(), dtype=TORCH_DT[dtype])
    qp = torch.empty((B, H, nt * nh * nw, D), device=dev(), dtype=TORCH_DT[dtype])
    ar.launch_q_prep(tx, qt, qp, T, LH, LW, *tile, nh, nw)
    back = torch.full_like(tx, float("nan"))
    ar.launch_untile(qt, back, T, LH, LW, *tile, nh, nw)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(to_np(back), x)
    np.testing.assert_array_equal(to_np(qp), O.block_mean(O.tile_raster(x, T, LH, LW, tile), dtype))


def test_strided_source_and_pool_only(cuda_ok):
    """HY passes q as a transposed view ([B,S,H,D] memory); pooling reads it in place."""
    B, S, H, D, T, LH, LW, tile = 2, 2 * 240, 4, 128, 2, 12, 20, (1, 8, 16)
    base, tbase = rand((B, S, H, D), 5, "bf16")
    view = tbase.transpose(1, 2)
    pool = K.pool_blocks(view, T, LH, LW, tile)
    torch.cuda.synchronize()
    ref = O.block_mean(O.tile_raster(base.transpose(0, 2, 1, 3), T, LH, LW, tile), "bf16")
    np.testing.assert_array_equal(to_np(pool), ref)


def test_frame_gather_fused_into_pooling(cuda_ok):
    B, H, D, F, LH, LW, tile = 1, 2, 128, 16, 10, 20, (4, 4, 8)
    x, tx = rand((B, H, F * LH * LW, D), 9, "bf16")
    ids = np.array([3, 15, 0, 7, 8, 2], np.int32)
    pool = K.pool_blocks(tx, len(ids), LH, LW, tile, frame_ids=torch.from_numpy(ids).to(dev()))
    torch.cuda.synchronize()
    g = O.gather_frames(x, ids, LH * LW)
    np.testing.assert_array_equal(to_np(pool), O.block_mean(O.tile_raster(g, len(ids), LH, LW, tile), "bf16"))


@pytest.mark.parametrize("dtype", ["bf16", "fp32"])
def test_gather_frames_bit_exact(cuda_ok, dtype):
    B, H, D, F, LH, LW = 2, 3, 128, 12, 30, 52
    x, tx = rand((B, H, F * LH * LW, D), 31, dtype)
    y, ty = rand((B, H, F * LH * LW, D), 32, dtype)
    ids = [11, 0, 5, 6, 3]
    k, v = memory.gather_kv(tx, ty, ids, (LH, LW))
    torch.cuda.synchronize()
    np.testing.assert_array_equal(to_np(k), O.gather_frames(x, ids, LH * LW))
    np.testing.assert_array_equal(to_np(v), O.gather_frames(y, ids, LH * LW))
    assert K.device_errors() == 0


def test_gather_frames_rejects_bad_frame_on_device(cuda_ok):
    x, tx = rand((1, 1, 4 * 64, 128), 3, "bf16")
    out = K.gather_frames(tx, torch.tensor([1, 9], dtype=torch.int32, device=dev()), 64)
    torch.cuda.synchronize()
    assert K.device_errors() & L.LI_DEVERR_BAD_INDEX
    np.testing.assert_array_equal(to_np(out[:, :, :64]), x[:, :, 64:128])
    assert (to_np(out[:, :, 64:]) == 0).all()


def test_text_blocks_zero_padded(cuda_ok):
    B, H, D, N, bs = 2, 2, 128, 130, 128
    kt, tkt = rand((B, H, N, D), 41, "bf16")
    vt, tvt = rand((B, H, N, D), 42, "bf16")
    ka = torch.full((B, H, 5, bs, D), float("nan"), device=dev(), dtype=torch.bfloat16)
    va = torch.full_like(ka, float("nan"))
    K.text_blocks(tkt, tvt, bs, ka, va)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(to_np(ka[:, :, :2]), O._text_blocks(kt, bs))
    np.testing.assert_array_equal(to_np(va[:, :, :2]), O._text_blocks(vt, bs))
    assert torch.isnan(ka[:, :, 2:].float()).all()


def test_prep_rejects_bad_arguments(cuda_ok):
    x = torch.zeros((1, 2, 100, 128), device=dev(), dtype=torch.bfloat16)
    with pytest.raises(ValueError):
        K.pool_blocks(x, 2, 8, 8, (1, 8, 8))  # 100 tokens is not a whole number of 8x8 frames
    y = torch.zeros((1, 2, 128, 128), device=dev(), dtype=torch.bfloat16)[..., 1:]
    with pytest.raises(ValueError):
        K.pool_blocks(y, 2, 8, 8, (1, 8, 8))  # D=127 rows are not 16-byte vectors


@pytest.mark.parametrize("dtype,D", [("bf16", 128), ("fp16", 64), ("fp32", 128)])
def test_pool_blocks_normalized_equals_normalize_after_pool(cuda_ok, dtype, D):
    """li_pool_blocks(normalized=1) == li_normalize_rows(li_pool_blocks(...)), bit for bit,
    with a frame list and a block offset into an existing pool."""
    B, H, T, LH, LW, tile = 1, 3, 8, 30, 52, (4, 4, 8)
    x, tx = rand((B, H, 10 * LH * LW, D), 321, dtype)
    ids = torch.tensor([9, 0, 3, 3, 7, 1, 2, 8], dtype=torch.int32, device=dev())
    nblk = 2 * 8 * 7
    raw = K.pool_blocks(tx, T, LH, LW, tile, frame_ids=ids)
    want = K.normalize_rows(raw)
    got = torch.full((B, H, nblk + 5, D), float("nan"), device=dev(), dtype=TORCH_DT[dtype])
    K.pool_blocks(tx, T, LH, LW, tile, frame_ids=ids, normalized=True, out=got, block_offset=5)
    torch.cuda.synchronize()
    assert torch.equal(got[:, :, 5:], want)
    assert torch.isnan(got[:, :, :5]).all()


@pytest.mark.parametrize("dtype", ["bf16", "fp32"])
def test_pool_blocks_multi_matches_separate_calls(cuda_ok, dtype):
    """One li_pool_blocks_multi launch over three jobs (different grids and tiles, a
    normalised pool, a fused frame gather, a block offset into a larger pool, a
    token-major strided source) writes exactly what three li_pool_blocks calls do."""
    D, LH, LW = 128 if dtype != "fp32" else 64, 10, 20
    HW = LH * LW
    _, q = rand((1, 3, 4 * HW, D), 871, dtype)
    _, kv = rand((6 * HW, 2, 3, D), 872, dtype)                      # token-major [L, 2, H, D]
    k = kv[:, 0].permute(1, 0, 2).unsqueeze(0)                         # [1, 3, L, D] strided view
    _, pool_src = rand((1, 3, 8 * HW, D), 873, dtype)
    ids = torch.tensor([6, 1, 3], dtype=torch.int32, device=dev())
    t1, t2 = (4, 4, 8), (1, 8, 16)
    nb = lambda T, t: int(np.prod(K.grid_blocks(T, LH, LW, t)))       # noqa: E731
    want = [K.pool_blocks(q, 4, LH, LW, t1, normalized=True),
            torch.zeros(1, 3, nb(6, t2) + 5, D, device=dev(), dtype=q.dtype),
            K.pool_blocks(pool_src, 3, LH, LW, t1, frame_ids=ids)]
    K.pool_blocks(k[:, :, 2 * HW:], 4, LH, LW, t2, out=want[1], block_offset=5 + nb(2, t2))
    got = [torch.empty_like(want[0]), torch.zeros_like(want[1]), torch.empty_like(want[2])]
    K.pool_blocks_multi([dict(src=q, T=4, LH=LH, LW=LW, tile=t1, out=got[0], normalized=True),
                         dict(src=k[:, :, 2 * HW:], T=4, LH=LH, LW=LW, tile=t2, out=got[1],
                              block_offset=5 + nb(2, t2)),
                         dict(src=pool_src, T=3, LH=LH, LW=LW, tile=t1, out=got[2], frame_ids=ids)])
    torch.cuda.synchronize()
    assert K.device_errors() == 0
    for g, w in zip(got, want):
        assert torch.equal(g, w)
