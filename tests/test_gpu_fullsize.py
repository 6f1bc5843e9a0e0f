"""GPU parity at the benchmark configurations' full sizes.

- Config 5 (the stack's layer: 24 heads, 64+4 frames of 30x52, tile (4,4,8),
  keep 25 %, cosine): full-size selection bit-exact against the oracle on every
  head, plus its size-independent invariants; attention with every block
  selected against torch fp32 attention over the same zero-padded tiled K/V;
  sparse attention against a torch fp32 reference on every head.
- Config 2 (HY decode, 16 heads, 4-frame chunk vs 16-frame context, tile
  (1,8,16), keep 25 %, recent_protect 4, scaled_dot_product) through the public
  ``run_sparse_attention``: selection bit-exact against the oracle and the output
  against a torch fp32 reference, every head.
- Config 3 end to end (MG, 24 heads): 16 retained frames gathered from a 64-frame
  K/V pool behind the current chunk, then the public ``run_sparse_attention``
  with ``q_block_offset`` (the query-chunk rows of the bidirectional selection),
  exactly as ``bench.py --workload mg_layer`` runs it: gather bit-exact, selection
  bit-exact against the oracle, output against a torch fp32 reference, every head.
- Config 4 (long-rollout sweep, HY shape, memory 8..64 frames, keep 10..100 %,
  lognormal per-key-block score bias): selection bit-exact against the oracle,
  attention against the torch fp32 reference.

The attention reference is plain torch fp32 (softmax over the selected blocks'
keys); the tolerance is the kernel's bf16 contract: max-abs 2e-2, mean-abs 2e-3.
"""

import math

import numpy as np
import pytest
import torch

from gpu_util import assert_close_bf16, dev
from light_interaction_project_b200 import _lib as L
from light_interaction_project_b200 import kernels as K
from oracle import li_oracle as O

pytestmark = pytest.mark.gpu


def _tiled(x, T, LH, LW, tile):
    """Zero-padded tiled copy [B, H, Nblk, bs, D] of a raster tensor (library tiling,
    itself bit-exact against the oracle in test_gpu_prep)."""
    B, H, _, D = x.shape
    nt, nh, nw = K.grid_blocks(T, LH, LW, tile)
    bs = tile[0] * tile[1] * tile[2]
    t = torch.empty(B, H, nt * nh * nw, bs, D, device=x.device, dtype=x.dtype)
    K.tile_pool(x, L.grid3d(T, LH, LW, tile), dst0=t)
    return t


def _valid_rows(q, T, LH, LW, tile):
    """[Nblk, bs] mask of the tiled rows that hold a real token (not padding)."""
    ones = torch.ones(1, 1, q.shape[2], 8, device=q.device, dtype=q.dtype)
    return _tiled(ones, T, LH, LW, tile)[0, 0, :, :, 0].bool()


def _ref_sparse(qt, kt, vt, idx, cnt, heads, scale):
    """fp32 attention of every query tile of `heads` over its selected blocks."""
    out = {}
    for h in heads:
        n = int(cnt[0, h, 0])
        assert bool((cnt[0, h] == n).all())
        sel = idx[0, h, :, :n].long()                                   # [nq, n]
        kk = kt[0, h].float()[sel].flatten(1, 2)                        # [nq, n*bs, D]
        vv = vt[0, h].float()[sel].flatten(1, 2)
        s = torch.bmm(qt[0, h].float(), kk.transpose(1, 2)) * scale     # [nq, bs, n*bs]
        out[h] = torch.bmm(torch.softmax(s, dim=-1), vv)                # [nq, bs, D]
    return out


def _pools_np(p):
    return p.float().cpu().numpy()


def test_config5_full_size(cuda_ok):
    LH, LW, tile, H, D, Fq, Fm = 30, 52, (4, 4, 8), 24, 128, 4, 64
    Fk = Fm + Fq
    bs = 128
    g = torch.Generator(device=dev()).manual_seed(55)
    q = torch.randn(1, H, Fq * LH * LW, D, generator=g, device=dev()).to(torch.bfloat16)
    k = torch.randn(1, H, Fk * LH * LW, D, generator=g, device=dev()).to(torch.bfloat16)
    v = torch.randn(1, H, Fk * LH * LW, D, generator=g, device=dev()).to(torch.bfloat16)
    gq, gk = K.grid_blocks(Fq, LH, LW, tile), K.grid_blocks(Fk, LH, LW, tile)
    nq, nk = 56, 952
    assert (int(np.prod(gq)), int(np.prod(gk))) == (nq, nk)

    # Selection at full size (normalised pools + dot, the pipeline's form).
    qp = K.normalize_rows(K.pool_blocks(q, Fq, LH, LW, tile))
    kp = K.normalize_rows(K.pool_blocks(k, Fk, LH, LW, tile))
    p = K.select_params(L.SELECT_BIDIR, "dot", tile, gk, gk, 0, 0, 0.25, 7, nk - nq)
    idx, cnt = K.select_blocks(qp, kp, p)
    torch.cuda.synchronize()
    S = O.prefill_budget(nk, 0.25)
    assert S == 238 and bool((cnt == S).all())
    sel = idx[..., :S]
    assert bool((sel[..., 1:] > sel[..., :-1]).all()), "lists sorted and unique"
    assert int(sel.min()) >= 0 and int(sel.max()) < nk
    # Protected 3D neighbours (distance <= 1 on the key grid) are always kept.
    nb = torch.from_numpy(O._neighbor_matrix(nq, nk, gk, nk - nq)).to(dev())      # [nq, nk]
    member = torch.zeros(1, H, nq, nk, dtype=torch.bool, device=dev())
    member.scatter_(3, sel.long(), True)
    assert bool((member | ~nb).all())
    # Bit-exact against the oracle on every head.
    ref_idx, ref_cnt = O.generate_prefill_indices(_pools_np(qp), _pools_np(kp), 0, gk,
                                                  dict(tile_size=tile, topk_ratio=0.25, sim_metric="dot"),
                                                  "bf16", q_offset=nk - nq)
    np.testing.assert_array_equal(idx.cpu().numpy(), ref_idx)
    np.testing.assert_array_equal(cnt.cpu().numpy(), ref_cnt)

    qt, kt, vt = _tiled(q, Fq, LH, LW, tile), _tiled(k, Fk, LH, LW, tile), _tiled(v, Fk, LH, LW, tile)
    scale = 1.0 / math.sqrt(D)

    # Every block selected: torch fp32 attention over the padded tiled K/V.
    all_idx = torch.arange(nk, device=dev(), dtype=torch.int32).expand(1, H, nq, nk).contiguous()
    all_cnt = torch.full((1, H, nq), nk, device=dev(), dtype=torch.int32)
    dense = K.sparse_attn_tiled(qt.flatten(2, 3), kt.flatten(2, 3), vt.flatten(2, 3), all_idx, all_cnt, bs)
    torch.cuda.synchronize()
    assert K.device_errors() == 0
    for h0 in range(0, H, 8):
        ref = torch.nn.functional.scaled_dot_product_attention(
            qt[:, h0:h0 + 8].flatten(2, 3).float(), kt[:, h0:h0 + 8].flatten(2, 3).float(),
            vt[:, h0:h0 + 8].flatten(2, 3).float())
        assert_close_bf16(dense[:, h0:h0 + 8].float().cpu().numpy(), ref.cpu().numpy(), what=f"dense heads {h0}+")

    # The selected lists through the fused raster kernel vs the fp32 reference.
    out = K.sparse_attn_raster(q, L.grid3d(Fq, LH, LW, tile), None, None, k, v, L.grid3d(Fk, LH, LW, tile), idx, cnt)
    out_t = _tiled(out, Fq, LH, LW, tile)
    torch.cuda.synchronize()
    assert K.device_errors() == 0
    valid = _valid_rows(q, Fq, LH, LW, tile)                                                  # [nq, bs]
    for h in range(H):
        r = _ref_sparse(qt, kt, vt, idx, cnt, (h,), scale)[h]
        assert_close_bf16(out_t[0, h][valid].float().cpu().numpy(), r[valid].cpu().numpy(), what=f"sparse head {h}")


@pytest.mark.parametrize("mem_frames,ratio", [(8, 0.10), (16, 0.25), (64, 0.25), (64, 1.0)])
def test_config4_sweep(cuda_ok, mem_frames, ratio):
    LH, LW, tile, H, D, Fq = 30, 52, (1, 8, 16), 2, 128, 4
    Fk = mem_frames
    params = dict(tile_size=tile, topk_ratio=ratio, recent_protect=4, sim_metric="scaled_dot_product")
    g = torch.Generator(device=dev()).manual_seed(100 + mem_frames)
    q = torch.randn(1, H, Fq * LH * LW, D, generator=g, device=dev()).to(torch.bfloat16)
    k = torch.randn(1, H, Fk * LH * LW, D, generator=g, device=dev()).to(torch.bfloat16)
    v = torch.randn(1, H, Fk * LH * LW, D, generator=g, device=dev()).to(torch.bfloat16)
    gq, gk = K.grid_blocks(Fq, LH, LW, tile), K.grid_blocks(Fk, LH, LW, tile)
    nq, nk = int(np.prod(gq)), int(np.prod(gk))
    rng = np.random.default_rng(7 + mem_frames)
    bias_np = (0.01 * rng.lognormal(0.0, 1.0, size=(1, 1, 1, nk))).astype(np.float32)
    bias = torch.from_numpy(bias_np).to(dev())

    qp = K.pool_blocks(q, Fq, LH, LW, tile)
    kp = K.pool_blocks(k, Fk, LH, LW, tile)
    p = K.select_params(L.SELECT_DECODE, "scaled_dot_product", tile, gq, gk, 0, 4, ratio)
    idx, cnt = K.select_blocks(qp, kp, p, score_bias=bias)
    torch.cuda.synchronize()
    ref_idx, ref_cnt = O.fast_generate_indices(_pools_np(qp), _pools_np(kp), 0, gq, gk, params, "bf16",
                                               score_bias=bias_np)
    np.testing.assert_array_equal(idx.cpu().numpy(), ref_idx)
    np.testing.assert_array_equal(cnt.cpu().numpy(), ref_cnt)

    out = K.sparse_attn_raster(q, L.grid3d(Fq, LH, LW, tile), None, None, k, v, L.grid3d(Fk, LH, LW, tile), idx, cnt)
    qt, kt, vt = _tiled(q, Fq, LH, LW, tile), _tiled(k, Fk, LH, LW, tile), _tiled(v, Fk, LH, LW, tile)
    out_t = _tiled(out, Fq, LH, LW, tile)
    torch.cuda.synchronize()
    assert K.device_errors() == 0
    ref = _ref_sparse(qt, kt, vt, idx, cnt, range(H), 1.0 / math.sqrt(D))
    valid = _valid_rows(q, Fq, LH, LW, tile)
    for h, r in ref.items():
        assert_close_bf16(out_t[0, h][valid].float().cpu().numpy(), r[valid].cpu().numpy(),
                          what=f"mem {mem_frames} ratio {ratio} head {h}")


def _sparse_raster_ref(q, k, v, idx, cnt, Fq, Fk, LH, LW, tile, out, what):
    """Every head of a raster-layout sparse attention against the torch fp32 reference."""
    qt, kt, vt = _tiled(q, Fq, LH, LW, tile), _tiled(k, Fk, LH, LW, tile), _tiled(v, Fk, LH, LW, tile)
    out_t = _tiled(out, Fq, LH, LW, tile)
    valid = _valid_rows(q, Fq, LH, LW, tile)
    scale = 1.0 / math.sqrt(q.shape[-1])
    for h in range(q.shape[1]):
        r = _ref_sparse(qt, kt, vt, idx, cnt, (h,), scale)[h]
        assert_close_bf16(out_t[0, h][valid].float().cpu().numpy(), r[valid].cpu().numpy(), what=f"{what} head {h}")


def test_config2_full_size_every_head(cuda_ok):
    from light_interaction_project_b200 import ar_sparse_operation as ar
    LH, LW, tile, H, D, Fq, Fk = 30, 52, (1, 8, 16), 16, 128, 4, 16
    params = dict(tile_size=tile, topk_ratio=0.25, recent_protect=4, sim_metric="scaled_dot_product")
    g = torch.Generator(device=dev()).manual_seed(22)
    q = torch.randn(1, H, Fq * LH * LW, D, generator=g, device=dev()).to(torch.bfloat16)
    k = torch.randn(1, H, Fk * LH * LW, D, generator=g, device=dev()).to(torch.bfloat16)
    v = torch.randn(1, H, Fk * LH * LW, D, generator=g, device=dev()).to(torch.bfloat16)
    empty = q[:, :, :0]
    out = ar.run_sparse_attention(q, empty, empty, k, v, 3, (LH, LW), params)
    gq, gk = K.grid_blocks(Fq, LH, LW, tile), K.grid_blocks(Fk, LH, LW, tile)
    qp, kp = K.pool_blocks(q, Fq, LH, LW, tile), K.pool_blocks(k, Fk, LH, LW, tile)
    idx, cnt = ar.fast_generate_indices(qp, kp, 0, gq, gk, params, dev())
    torch.cuda.synchronize()
    assert K.device_errors() == 0
    ref_idx, ref_cnt = O.fast_generate_indices(_pools_np(qp), _pools_np(kp), 0, gq, gk, params, "bf16")
    np.testing.assert_array_equal(idx.cpu().numpy(), ref_idx)
    np.testing.assert_array_equal(cnt.cpu().numpy(), ref_cnt)
    assert idx.shape[-1] == 112
    _sparse_raster_ref(q, k, v, idx, cnt, Fq, Fk, LH, LW, tile, out, "config 2")


def test_config3_end_to_end_with_gather(cuda_ok):
    from light_interaction_project_b200 import bi_sparse_operation as mg
    LH, LW, tile, H, D, Fq, Fmem, Fpool = 30, 52, (4, 4, 8), 24, 128, 4, 16, 64
    HW = LH * LW
    Fk = Fmem + Fq
    params = dict(tile_size=tile, topk_ratio=0.30, sim_metric="cosine")
    g = torch.Generator(device=dev()).manual_seed(33)
    k_pool = torch.randn(1, H, Fpool * HW, D, generator=g, device=dev()).to(torch.bfloat16)
    v_pool = torch.randn(1, H, Fpool * HW, D, generator=g, device=dev()).to(torch.bfloat16)
    ids_np = np.random.default_rng(1234).choice(Fpool, Fmem, replace=False).astype(np.int32)
    ids = torch.from_numpy(ids_np).to(dev())
    k_buf = torch.randn(1, H, Fk * HW, D, generator=g, device=dev()).to(torch.bfloat16)
    v_buf = torch.randn(1, H, Fk * HW, D, generator=g, device=dev()).to(torch.bfloat16)
    q = torch.randn(1, H, Fq * HW, D, generator=g, device=dev()).to(torch.bfloat16)
    gk = K.grid_blocks(Fk, LH, LW, tile)
    nq, nk = 56, 280
    assert int(np.prod(gk)) == nk
    # The benchmark's call: gather 16 of the pool's 64 frames ahead of the current
    # chunk, then the MG operator on the query chunk's rows.
    K.gather_frames(k_pool, ids, HW, out=k_buf[:, :, :Fmem * HW])
    K.gather_frames(v_pool, ids, HW, out=v_buf[:, :, :Fmem * HW])
    out = mg.run_sparse_attention(q, k_buf, v_buf, 0, 0, (LH, LW), params, q_block_offset=nk - nq)
    torch.cuda.synchronize()
    assert K.device_errors() == 0
    sel = torch.from_numpy(ids_np.astype(np.int64)).to(dev())
    want_k = k_pool.view(1, H, Fpool, HW, D)[:, :, sel].reshape(1, H, Fmem * HW, D)
    want_v = v_pool.view(1, H, Fpool, HW, D)[:, :, sel].reshape(1, H, Fmem * HW, D)
    assert torch.equal(k_buf[:, :, :Fmem * HW], want_k) and torch.equal(v_buf[:, :, :Fmem * HW], want_v)
    # Selection: the operator's own pools and indices against the oracle.
    qp = K.pool_blocks(q, Fq, LH, LW, tile)
    kp = K.pool_blocks(k_buf, Fk, LH, LW, tile)
    idx, cnt = mg.generate_prefill_indices(qp, kp, 0, gk, params, dev(), q_block_offset=nk - nq)
    ref_idx, ref_cnt = O.generate_prefill_indices(_pools_np(qp), _pools_np(kp), 0, gk, params, "bf16",
                                                  q_offset=nk - nq)
    np.testing.assert_array_equal(idx.cpu().numpy(), ref_idx)
    np.testing.assert_array_equal(cnt.cpu().numpy(), ref_cnt)
    assert idx.shape[-1] == 84
    _sparse_raster_ref(q, k_buf, v_buf, idx, cnt, Fq, Fk, LH, LW, tile, out, "config 3")
