"""GPU parity: block selection is bit-exact with the oracle (ranking scores and
indices), and its ranking step reproduces torch's own CUDA ``topk`` + ``sort``."""

import math

import numpy as np
import pytest
import torch

from golden_util import list_cases, load_case, tie_explained
from gpu_util import TORCH_DT, dev, rand, to_gpu, to_np
from light_interaction_project_b200 import _lib as L
from light_interaction_project_b200 import ar_sparse_operation as ar
from light_interaction_project_b200 import bi_sparse_operation as mg
from light_interaction_project_b200 import bi_sparse_operation_for_KV_cache as hyp
from light_interaction_project_b200 import kernels as K
from oracle import li_oracle as O

pytestmark = pytest.mark.gpu

DECODE_CASES = [
    # (dtype, metric, grid_q, grid_k, tile, text_len, recent_protect, ratio, quant)
    ("bf16", "scaled_dot_product", (4, 4, 4), (16, 4, 4), (1, 8, 16), 0, 4, 0.25, None),
    ("bf16", "cosine", (1, 8, 7), (5, 8, 7), (4, 4, 8), 77, 4, 0.175, None),
    ("bf16", "dot", (2, 2, 3), (9, 2, 3), (4, 8, 4), 300, 2, 0.5, 4),
    ("fp16", "scaled_dot_product", (1, 2, 2), (6, 2, 2), (2, 4, 8), 3, 2, 0.1, None),
    ("fp32", "scaled_dot_product", (1, 2, 1), (3, 2, 1), (2, 4, 8), 0, 2, 0.5, None),
    ("bf16", "cosine", (1, 1, 2), (1, 1, 2), (1, 8, 16), 0, 9, 0.3, None),   # protect > available
    ("bf16", "scaled_dot_product", (1, 4, 4), (64, 4, 4), (1, 8, 16), 0, 1, 0.1, 2),  # 1024 key blocks
    # 3040 key blocks (12 per top-k thread, not a multiple of 256), quantised: ties span thread slices
    ("bf16", "scaled_dot_product", (1, 4, 4), (190, 4, 4), (1, 8, 16), 0, 1, 0.1, 2),
    # 2800 key blocks with 32-bit radix keys (four 8-bit passes)
    ("fp32", "dot", (1, 2, 2), (700, 2, 2), (2, 4, 8), 0, 2, 0.3, 4),
]


def _pools(seed, B, H, nq, nk, D, dtype, quant):
    qp, _ = rand((B, H, nq, D), seed, dtype, scale=0.3)
    kp, _ = rand((B, H, nk, D), seed + 1, dtype, scale=0.3)
    if quant:
        qp = O.round_to(np.round(qp * quant) / quant, dtype)
        kp = O.round_to(np.round(kp * quant) / quant, dtype)
    return qp, kp


@pytest.mark.parametrize("case", DECODE_CASES)
def test_decode_selection_bit_exact(cuda_ok, case):
    dtype, metric, gq, gk, tile, text_len, rp, ratio, quant = case
    B, H, D = 1, 3, 128 if dtype != "fp32" else 64
    nq, nk = int(np.prod(gq)), int(np.prod(gk))
    qp, kp = _pools(123, B, H, nq, nk, D, dtype, quant)
    params = dict(tile_size=tile, sim_metric=metric, recent_protect=rp, topk_ratio=ratio)
    ref_idx, ref_cnt, ref_rank = O.fast_generate_indices(qp, kp, text_len, gq, gk, params, dtype, return_scores=True)
    p = K.select_params(L.SELECT_DECODE, metric, tile, gq, gk, text_len, rp, ratio)
    idx, cnt, rank = K.select_blocks(to_gpu(qp, dtype), to_gpu(kp, dtype), p, return_rank=True)
    np.testing.assert_array_equal(to_np(rank), ref_rank)
    np.testing.assert_array_equal(idx.cpu().numpy(), ref_idx)
    np.testing.assert_array_equal(cnt.cpu().numpy(), ref_cnt)
    # The reference-named entry point gives the same result.
    idx2, cnt2 = ar.fast_generate_indices(to_gpu(qp, dtype), to_gpu(kp, dtype), text_len, gq, gk, params, dev())
    assert torch.equal(idx2, idx) and torch.equal(cnt2, cnt)


BIDIR_CASES = [
    ("bf16", "cosine", (5, 8, 7), (4, 4, 8), 0, 0.3, None, None),
    ("bf16", "scaled_dot_product", (4, 4, 4), (4, 8, 4), 13, 0.3, 2, None),
    ("bf16", "cosine", (20, 8, 7), (4, 4, 8), 0, 0.3, None, 56 * 16),   # config-3 query-chunk rows
    ("fp16", "dot", (1, 2, 3), (4, 4, 8), 0, 0.5, None, None),            # budget floor of 7 clamps to N_k
    ("fp32", "cosine", (2, 3, 2), (2, 4, 8), 200, 0.25, None, None),
]


@pytest.mark.parametrize("case", BIDIR_CASES)
def test_bidir_selection_bit_exact(cuda_ok, case):
    dtype, metric, gk, tile, text_len, ratio, quant, q_off = case
    B, H, D = 2, 2, 128 if dtype != "fp32" else 64
    nk = int(np.prod(gk))
    nq = nk if q_off is None else nk - q_off
    qp, kp = _pools(321, B, H, nq, nk, D, dtype, quant)
    params = dict(tile_size=tile, sim_metric=metric, topk_ratio=ratio)
    ref_idx, ref_cnt, ref_rank = O.generate_prefill_indices(qp, kp, text_len, gk, params, dtype,
                                                            q_offset=q_off, return_scores=True)
    p = K.select_params(L.SELECT_BIDIR, metric, tile, gk, gk, text_len, 0, ratio, 7, q_off or 0)
    idx, cnt, rank = K.select_blocks(to_gpu(qp, dtype), to_gpu(kp, dtype), p, return_rank=True)
    np.testing.assert_array_equal(to_np(rank), ref_rank)
    np.testing.assert_array_equal(idx.cpu().numpy(), ref_idx)
    np.testing.assert_array_equal(cnt.cpu().numpy(), ref_cnt)
    if q_off is None:
        for fn in (mg.generate_prefill_indices, hyp.generate_prefill_indices):
            i2, c2 = fn(to_gpu(qp, dtype), to_gpu(kp, dtype), text_len, gk, params, dev())
            assert torch.equal(i2, idx) and torch.equal(c2, cnt)


def test_bidir_requires_square_like_reference(cuda_ok):
    qp = torch.zeros((1, 1, 4, 128), device=dev(), dtype=torch.bfloat16)
    kp = torch.zeros((1, 1, 8, 128), device=dev(), dtype=torch.bfloat16)
    with pytest.raises(RuntimeError):
        mg.generate_prefill_indices(qp, kp, 0, (2, 2, 2), dict(tile_size=(4, 4, 8), topk_ratio=0.3), dev())


@pytest.mark.parametrize("name", [c for c in list_cases() if "pool" not in c])
def test_selection_on_reference_fixture_pools(cuda_ok, name):
    """The reference's own pooled tensors in; indices equal the reference's
    except exactly-tied boundary scores, and equal the oracle's bit for bit."""
    meta, g = load_case(name)
    dtype = meta["dtype"]
    params = dict(meta["params"])
    params["tile_size"] = tuple(params["tile_size"])
    tile = params["tile_size"]
    bs = math.prod(tile)
    ntxt = (meta["text_len"] + bs - 1) // bs
    qp, kp = to_gpu(g["q_pool"], dtype), to_gpu(g["k_pool"], dtype)
    kind = meta["kind"]
    if kind in ("hy_decode", "selection_decode"):
        if kind == "hy_decode":
            gq = O.grid_dims(meta["Fq"], meta["LH"], meta["LW"], tile)
            gk = O.grid_dims(meta["Fk"], meta["LH"], meta["LW"], tile)
        else:
            gq, gk = meta["grid_q"], meta["grid_k"]
        idx, cnt = ar.fast_generate_indices(qp, kp, meta["text_len"], gq, gk, params, dev())
        oi, oc = O.fast_generate_indices(g["q_pool"], g["k_pool"], meta["text_len"], gq, gk, params, dtype)
    else:
        gk = meta.get("grid_k") or O.grid_dims(meta["Fk"], meta["LH"], meta["LW"], tile)
        fn = hyp.generate_prefill_indices if kind in ("hy_prefill", "selection_bidir_hy") else mg.generate_prefill_indices
        idx, cnt = fn(qp, kp, meta["text_len"], gk, params, dev())
        oi, oc = O.generate_prefill_indices(g["q_pool"], g["k_pool"], meta["text_len"], gk, params, dtype)
    idx, cnt = idx.cpu().numpy(), cnt.cpu().numpy()
    np.testing.assert_array_equal(idx, oi)
    np.testing.assert_array_equal(cnt, g["counts"])
    same = (idx == g["indices"]).all(-1)
    for i in zip(*np.nonzero(~same)):
        assert tie_explained(g["indices"][i], idx[i], g["rank_scores"][i], dtype, ntxt), (name, i)


@pytest.mark.parametrize("dtype", ["bf16", "fp16", "fp32"])
def test_rank_matches_torch_cuda_topk(cuda_ok, dtype):
    """Ranking step vs torch.topk + torch.sort on the GPU, on tie-heavy scores
    (values on a coarse grid, signed zeros included)."""
    B, H, nq, nk, k = 2, 3, 40, 300, 77
    rng = np.random.default_rng(7)
    s = rng.integers(-6, 7, size=(B, H, nq, nk)).astype(np.float32) / 4.0
    s[..., ::17] = -0.0
    t = torch.from_numpy(s).to(dev()).to(TORCH_DT[dtype])
    _, ti = torch.topk(t, k=k, dim=-1)
    ti, _ = torch.sort(ti, dim=-1)
    idx, cnt = K.rank_blocks(t.float(), TORCH_DT[dtype], k, 130, 128)
    assert torch.equal(idx[..., :2].cpu(), torch.arange(2, dtype=torch.int32).expand(B, H, nq, 2))
    assert torch.equal(idx[..., 2:].long().cpu() - 2, ti.cpu())
    assert (cnt == 2 + k).all()


@pytest.mark.parametrize("dtype", ["bf16", "fp16", "fp32"])
def test_normalize_rows_and_cosine_equals_dot_of_normalised(cuda_ok, dtype):
    """li_normalize_rows is bit-exact with the oracle's F.normalize, and cosine
    selection equals plain-dot selection of the normalised pools (the pipeline's path)."""
    B, H, nq, nk, D = 1, 3, 56, 280, 128 if dtype != "fp32" else 64
    qp, _ = rand((B, H, nq, D), 77, dtype, scale=0.3)
    kp, _ = rand((B, H, nk, D), 78, dtype, scale=0.3)
    tq, tk = to_gpu(qp, dtype), to_gpu(kp, dtype)
    nqn = K.normalize_rows(tq)
    np.testing.assert_array_equal(to_np(nqn), O.normalize_rows(qp, dtype))
    gk = (5, 8, 7)
    p_cos = K.select_params(L.SELECT_BIDIR, "cosine", (4, 4, 8), gk, gk, 0, 0, 0.3, 7, nk - nq)
    p_dot = K.select_params(L.SELECT_BIDIR, "dot", (4, 4, 8), gk, gk, 0, 0, 0.3, 7, nk - nq)
    i1, c1, r1 = K.select_blocks(tq, tk, p_cos, return_rank=True)
    i2, c2, r2 = K.select_blocks(nqn, K.normalize_rows(tk), p_dot, return_rank=True)
    assert torch.equal(i1, i2) and torch.equal(c1, c2) and torch.equal(r1, r2)


@pytest.mark.parametrize("mode", ["decode", "bidir"])
def test_two_kernel_and_single_kernel_paths_agree(cuda_ok, mode):
    """With a workspace the scores and the top-k run as two kernels; without,
    as one. Both follow the same arithmetic: identical indices and scores."""
    dtype = "bf16"
    B, H, D = 1, 4, 128
    gk = (17, 8, 7)
    nk = int(np.prod(gk))
    nq = 56
    qp, kp = _pools(55, B, H, nq, nk, D, dtype, None)
    tq, tk = to_gpu(qp, dtype), to_gpu(kp, dtype)
    if mode == "decode":
        p = K.select_params(L.SELECT_DECODE, "scaled_dot_product", (4, 4, 8), (1, 8, 7), gk, 5, 4, 0.25)
    else:
        p = K.select_params(L.SELECT_BIDIR, "cosine", (4, 4, 8), gk, gk, 0, 0, 0.25, 7, nk - nq)
    i1, c1, r1 = K.select_blocks(tq, tk, p, return_rank=True, use_workspace=True)
    i2, c2, r2 = K.select_blocks(tq, tk, p, return_rank=True, use_workspace=False)
    assert torch.equal(i1, i2) and torch.equal(c1, c2) and torch.equal(r1, r2)
