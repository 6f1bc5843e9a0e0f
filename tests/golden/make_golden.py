"""Generate the golden fixtures by running the reference's own code on CPU.

Run in the build container, where the reference checkout is readable:

    python tests/golden/make_golden.py --ref-root PATH   (or LI_REFERENCE_ROOT=PATH)

It imports the reference's sparse-attention modules unchanged (a small package
shim satisfies their relative imports; ``hyvideo.commons.infer_state`` is
stubbed), runs their Triton prep / attention / untile kernels under
``TRITON_INTERPRET=1`` and their torch selection functions as is, and writes one
``.npz`` per case next to this file. Inputs are not stored: they are rebuilt
from seeds by ``oracle.inputs`` (bit-reproducible), and each fixture stores a
checksum of them. Captured per case:

* ``q_pool`` / ``k_pool`` — written by the reference's Triton prep kernels;
* ``rank_scores`` — the exact tensor the reference passed to ``torch.topk``
  (captured by wrapping ``torch.topk``), so selection can be checked on the
  reference's own scores;
* ``indices`` / ``counts`` — the reference's selection output;
* ``out_ref`` — the reference orchestrator's output (its Triton attention);
* ``out_masked`` — dense masked fp32 attention with the reference's indices
  (the reference CPU path of the toy configuration).

Nothing on the GPU box runs this script; the fixtures it writes travel instead.
"""

from __future__ import annotations

import argparse
import hashlib
import importlib
import json
import math
import os
import sys
import types

os.environ.setdefault("TRITON_INTERPRET", "1")

import numpy as np  # noqa: E402
import torch  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)

from oracle.inputs import det_normal_like  # noqa: E402
from oracle import li_oracle  # noqa: E402


def _patch_triton_interpreter():
    """Make the Triton CPU interpreter's bf16 arithmetic match the GPU's.

    The interpreter that ships with triton 3.6.0 emulates bf16 in two wrong
    ways. (a) It truncates fp32 -> bf16 casts (``_convert_float`` with no
    rounding mode), where compiled Triton lowers ``.to(tl.bfloat16)`` to an
    LLVM ``fptrunc``, which rounds to nearest even. (b) ``create_dot`` feeds the
    uint16 storage of bf16 operands straight into ``np.matmul``, which multiplies
    the bit patterns as integers. Both routines are replaced here with exact
    bf16 <-> fp32 conversions and an fp32 matmul. The reference's kernels are
    not touched.
    """
    import triton.language as tl
    from triton.runtime import interpreter as itp

    def f32_to_bf16_bits(x):
        u = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
        r = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
        return r.astype(np.uint16)

    def bf16_bits_to_f32(b):
        return (np.asarray(b).astype(np.uint32) << 16).view(np.float32)

    orig_cast = itp.InterpreterBuilder.cast_impl
    orig_fp = itp.InterpreterBuilder.create_fp_to_fp
    orig_dot = itp.InterpreterBuilder.create_dot

    def cast_impl(self, src, dst_type):
        s, d = src.dtype.scalar, dst_type.scalar
        if s == tl.float32 and d == tl.bfloat16:
            return itp.TensorHandle(f32_to_bf16_bits(src.data), d)
        if s == tl.bfloat16 and d == tl.float32:
            return itp.TensorHandle(bf16_bits_to_f32(src.data), d)
        return orig_cast(self, src, dst_type)

    def create_fp_to_fp(self, src, dst_type, rounding_mode):
        if src.dtype.scalar == tl.float32 and dst_type.scalar == tl.bfloat16:
            return itp.TensorHandle(f32_to_bf16_bits(src.data), dst_type.scalar)
        return orig_fp(self, src, dst_type, rounding_mode)

    def create_dot(self, a, b, d, input_precision, max_num_imprecise_acc):
        if a.dtype.scalar == tl.bfloat16 or b.dtype.scalar == tl.bfloat16:
            a32 = bf16_bits_to_f32(a.data) if a.dtype.scalar == tl.bfloat16 else a.data.astype(np.float32)
            b32 = bf16_bits_to_f32(b.data) if b.dtype.scalar == tl.bfloat16 else b.data.astype(np.float32)
            return itp.TensorHandle(np.matmul(a32, b32, dtype=np.float32) + d.data, d.dtype.scalar)
        return orig_dot(self, a, b, d, input_precision, max_num_imprecise_acc)

    itp.InterpreterBuilder.cast_impl = cast_impl
    itp.InterpreterBuilder.create_fp_trunc = lambda self, src, dst_type: cast_impl(self, src, dst_type)
    itp.InterpreterBuilder.create_fp_ext = lambda self, src, dst_type: cast_impl(self, src, dst_type)
    itp.InterpreterBuilder.create_fp_to_fp = create_fp_to_fp
    itp.InterpreterBuilder.create_dot = create_dot


def _load_reference(ref_root):
    _patch_triton_interpreter()
    hy_dir = os.path.join(ref_root, "hy-worldplay/files/hyvideo/models/transformers/modules")
    mg_dir = os.path.join(ref_root, "matrix-game-3.0/files/wan/modules")
    state = types.SimpleNamespace(current_chunk_index=0)
    # Stub for ``from hyvideo.commons.infer_state import get_infer_state``.
    for name in ("hyvideo", "hyvideo.commons"):
        m = types.ModuleType(name)
        m.__path__ = []
        sys.modules[name] = m
    inf = types.ModuleType("hyvideo.commons.infer_state")
    inf.get_infer_state = lambda: state
    sys.modules["hyvideo.commons.infer_state"] = inf
    mods = {}
    for pkg, d in (("liref_hy", hy_dir), ("liref_mg", mg_dir)):
        p = types.ModuleType(pkg)
        p.__path__ = [d]
        sys.modules[pkg] = p
    mods["hy_ar"] = importlib.import_module("liref_hy.ar_sparse_operation")
    mods["hy_pre"] = importlib.import_module("liref_hy.bi_sparse_operation_for_KV_cache")
    mods["mg"] = importlib.import_module("liref_mg.bi_sparse_operation")
    for k in ("hy_ar", "hy_pre", "mg"):
        assert mods[k].HAS_TRITON, "reference Triton path did not import"
    return mods, state


class _TopkRecorder:
    """Wraps ``torch.topk`` to keep the last ranking tensor the reference used."""

    def __init__(self):
        self.last = None
        self._orig = torch.topk

    def __enter__(self):
        def rec(inp, *a, **kw):
            self.last = inp.detach().clone()
            return self._orig(inp, *a, **kw)
        torch.topk = rec
        return self

    def __exit__(self, *exc):
        torch.topk = self._orig


def _t(x, dtype):
    t = torch.from_numpy(np.ascontiguousarray(x, np.float32))
    return t.to(torch.bfloat16) if dtype == "bf16" else t


def _np(t):
    return t.detach().to(torch.float32).cpu().numpy()


def _checksum(*arrays):
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a, np.float32).tobytes())
    return h.hexdigest()


def _pools_via_reference(mod, q, k_vis, v_vis, text_len, latent_hw, tile, dtype):
    """Run the reference's own prep kernels to get its pooled tensors."""
    LH, LW = latent_hw
    tt, th, tw = tile
    bs = tt * th * tw
    nh, nw = (LH + th - 1) // th, (LW + tw - 1) // tw
    T_q, T_k = q.shape[2] // (LH * LW), k_vis.shape[2] // (LH * LW)
    nt_q, nt_k = (T_q + tt - 1) // tt, (T_k + tt - 1) // tt
    ntxt = (text_len + bs - 1) // bs
    B, H, _, D = q.shape
    qt = torch.empty((B, H, nt_q * nh * nw, bs, D), dtype=q.dtype)
    qp = torch.empty((B, H, nt_q * nh * nw, D), dtype=q.dtype)
    ka = torch.empty((B, H, ntxt + nt_k * nh * nw, bs, D), dtype=q.dtype)
    va = torch.empty_like(ka)
    kp = torch.empty((B, H, nt_k * nh * nw, D), dtype=q.dtype)
    mod.launch_q_prep(q, qt, qp, T_q, LH, LW, tt, th, tw, nh, nw)
    mod.launch_kv_prep(k_vis, v_vis, ka, va, kp, ntxt, 0, T_k, LH, LW, tt, th, tw, nh, nw)
    return qt, qp, ka, va, kp, (nt_q, nh, nw), (nt_k, nh, nw)


def _masked(qt, ka, va, idx, cnt, text_k=None):
    return li_oracle.dense_masked_attention(_np(qt), _np(ka), _np(va), idx, cnt)


def case_hy_decode(mods, name, seed, dtype, B, H, D, LH, LW, Fq, Fk, text_len, params):
    """HY decode: ``run_sparse_attention`` (ar_sparse_operation.py:289-362)."""
    m = mods["hy_ar"]
    HW = LH * LW
    q = det_normal_like((B, H, Fq * HW, D), seed + 0, dtype)
    kt = det_normal_like((B, H, text_len, D), seed + 1, dtype)
    vt = det_normal_like((B, H, text_len, D), seed + 2, dtype)
    kv = det_normal_like((B, H, Fk * HW, D), seed + 3, dtype)
    vv = det_normal_like((B, H, Fk * HW, D), seed + 4, dtype)
    tq, tkt, tvt, tkv, tvv = (_t(a, dtype) for a in (q, kt, vt, kv, vv))
    with _TopkRecorder() as rec:
        out = m.run_sparse_attention(tq, tkt, tvt, tkv, tvv, 5, (LH, LW), params)
    qt, qp, ka, va, kp, gq, gk = _pools_via_reference(m, tq, tkv, tvv, text_len, (LH, LW),
                                                      params["tile_size"], dtype)
    bs = math.prod(params["tile_size"])
    ntxt = (text_len + bs - 1) // bs
    if ntxt:
        pad = ntxt * bs - text_len
        ka[:, :, :ntxt] = torch.nn.functional.pad(tkt, (0, 0, 0, pad)).view(B, H, ntxt, bs, D)
        va[:, :, :ntxt] = torch.nn.functional.pad(tvt, (0, 0, 0, pad)).view(B, H, ntxt, bs, D)
    idx, cnt = m.fast_generate_indices(qp, kp, text_len, gq, gk, params, "cpu")
    idx, cnt = idx.numpy(), cnt.numpy()
    return dict(
        kind="hy_decode", inputs_sha=_checksum(q, kt, vt, kv, vv),
        q_pool=_np(qp), k_pool=_np(kp), rank_scores=_np(rec.last), indices=idx, counts=cnt,
        out_ref=_np(out), out_masked=li_oracle.untile_raster(
            _masked(qt, ka, va, idx, cnt), Fq, LH, LW, params["tile_size"]),
        meta=dict(seed=seed, dtype=dtype, B=B, H=H, D=D, LH=LH, LW=LW, Fq=Fq, Fk=Fk,
                  text_len=text_len, params={k: (list(v) if isinstance(v, tuple) else v)
                                             for k, v in params.items()}))


def case_hy_prefill(mods, state, name, seed, dtype, B, H, D, LH, LW, F, text_len, params):
    """HY prefill: ``run_sparse_prefill_attention`` (bi_sparse_operation_for_KV_cache.py:301-395)."""
    m = mods["hy_pre"]
    state.current_chunk_index = 3
    HW = LH * LW
    q = det_normal_like((B, H, F * HW, D), seed + 0, dtype)
    kt = det_normal_like((B, H, text_len, D), seed + 1, dtype)
    vt = det_normal_like((B, H, text_len, D), seed + 2, dtype)
    kv = det_normal_like((B, H, F * HW, D), seed + 3, dtype)
    vv = det_normal_like((B, H, F * HW, D), seed + 4, dtype)
    tq, tkt, tvt, tkv, tvv = (_t(a, dtype) for a in (q, kt, vt, kv, vv))
    with _TopkRecorder() as rec:
        out = m.run_sparse_prefill_attention(tq, tkt, tvt, tkv, tvv, 5, (LH, LW), params)
    qt, qp, ka, va, kp, gq, gk = _pools_via_reference(m, tq, tkv, tvv, text_len, (LH, LW),
                                                      params["tile_size"], dtype)
    bs = math.prod(params["tile_size"])
    ntxt = (text_len + bs - 1) // bs
    if ntxt:
        pad = ntxt * bs - text_len
        ka[:, :, :ntxt] = torch.nn.functional.pad(tkt, (0, 0, 0, pad)).view(B, H, ntxt, bs, D)
        va[:, :, :ntxt] = torch.nn.functional.pad(tvt, (0, 0, 0, pad)).view(B, H, ntxt, bs, D)
    idx, cnt = m.generate_prefill_indices(qp, kp, text_len, gk, params, "cpu")
    idx, cnt = idx.numpy(), cnt.numpy()
    state.current_chunk_index = 0
    return dict(
        kind="hy_prefill", inputs_sha=_checksum(q, kt, vt, kv, vv),
        q_pool=_np(qp), k_pool=_np(kp), rank_scores=_np(rec.last), indices=idx, counts=cnt,
        out_ref=_np(out), out_masked=li_oracle.untile_raster(
            _masked(qt, ka, va, idx, cnt), F, LH, LW, params["tile_size"]),
        meta=dict(seed=seed, dtype=dtype, B=B, H=H, D=D, LH=LH, LW=LW, Fq=F, Fk=F,
                  text_len=text_len, params={k: (list(v) if isinstance(v, tuple) else v)
                                             for k, v in params.items()}))


def case_mg(mods, name, seed, dtype, B, H, D, LH, LW, F, text_len, params):
    """MG: ``run_sparse_attention(q, k, v, text_len, ...)`` (bi_sparse_operation.py:236-348)."""
    m = mods["mg"]
    HW = LH * LW
    q = det_normal_like((B, H, F * HW, D), seed + 0, dtype)
    k = det_normal_like((B, H, text_len + F * HW, D), seed + 3, dtype)
    v = det_normal_like((B, H, text_len + F * HW, D), seed + 4, dtype)
    tq, tk, tv = (_t(a, dtype) for a in (q, k, v))
    with _TopkRecorder() as rec:
        out = m.run_sparse_attention(tq, tk, tv, text_len, 5, (LH, LW), params)
    qt, qp, ka, va, kp, gq, gk = _pools_via_reference(
        m, tq, tk[:, :, text_len:], tv[:, :, text_len:], text_len, (LH, LW),
        params["tile_size"], dtype)
    bs = math.prod(params["tile_size"])
    ntxt = (text_len + bs - 1) // bs
    if ntxt:
        pad = ntxt * bs - text_len
        ka[:, :, :ntxt] = torch.nn.functional.pad(tk[:, :, :text_len], (0, 0, 0, pad)).view(B, H, ntxt, bs, D)
        va[:, :, :ntxt] = torch.nn.functional.pad(tv[:, :, :text_len], (0, 0, 0, pad)).view(B, H, ntxt, bs, D)
    idx, cnt = m.generate_prefill_indices(qp, kp, text_len, gk, params, "cpu")
    idx, cnt = idx.numpy(), cnt.numpy()
    return dict(
        kind="mg", inputs_sha=_checksum(q, k, v),
        q_pool=_np(qp), k_pool=_np(kp), rank_scores=_np(rec.last), indices=idx, counts=cnt,
        out_ref=_np(out), out_masked=li_oracle.untile_raster(
            _masked(qt, ka, va, idx, cnt), F, LH, LW, params["tile_size"]),
        meta=dict(seed=seed, dtype=dtype, B=B, H=H, D=D, LH=LH, LW=LW, Fq=F, Fk=F,
                  text_len=text_len, params={k: (list(v) if isinstance(v, tuple) else v)
                                             for k, v in params.items()}))


def case_selection(mods, name, seed, dtype, mode, B, H, D, grid_q, grid_k, text_len, params,
                   quant=None):
    """Selection only, on seeded pools; ``quant`` snaps values to a coarse grid to
    force exact score ties."""
    nq = int(np.prod(grid_q))
    nk = int(np.prod(grid_k))
    qp = det_normal_like((B, H, nq, D), seed, dtype, scale=0.2)
    kp = det_normal_like((B, H, nk, D), seed + 1, dtype, scale=0.2)
    if quant:
        qp = li_oracle.round_to(np.round(qp * quant) / quant, dtype)
        kp = li_oracle.round_to(np.round(kp * quant) / quant, dtype)
    tq, tk = _t(qp, dtype), _t(kp, dtype)
    with _TopkRecorder() as rec:
        if mode == "decode":
            idx, cnt = mods["hy_ar"].fast_generate_indices(tq, tk, text_len, grid_q, grid_k, params, "cpu")
        elif mode == "bidir_hy":
            idx, cnt = mods["hy_pre"].generate_prefill_indices(tq, tk, text_len, grid_k, params, "cpu")
        else:
            idx, cnt = mods["mg"].generate_prefill_indices(tq, tk, text_len, grid_k, params, "cpu")
    return dict(
        kind="selection_" + mode, inputs_sha=_checksum(qp, kp), q_pool=qp, k_pool=kp,
        rank_scores=_np(rec.last), indices=idx.numpy(), counts=cnt.numpy(),
        meta=dict(seed=seed, dtype=dtype, B=B, H=H, D=D, mode=mode, grid_q=list(grid_q),
                  grid_k=list(grid_k), text_len=text_len, quant=quant,
                  params={k: (list(v) if isinstance(v, tuple) else v) for k, v in params.items()}))


CASES = {
    # BASELINE config 1 (toy): fp32, H4, D64, 8x8 latent, 3 chunks of 2 frames,
    # query = last chunk, KV = all 6 frames, tile (2,4,8) = 64 tokens, protect the
    # query's own chunk (2 frames) + top-k 2 of 4 history blocks.
    "toy_decode_fp32": lambda M, S: case_hy_decode(
        M, "toy", 0, "fp32", 1, 4, 64, 8, 8, 2, 6, 0,
        dict(tile_size=(2, 4, 8), topk_ratio=0.5, recent_protect=2, sim_metric="scaled_dot_product")),
    "hy_decode_bf16_text": lambda M, S: case_hy_decode(
        M, "hyd", 100, "bf16", 1, 2, 128, 12, 20, 2, 6, 5,
        dict(tile_size=(1, 8, 16), topk_ratio=0.25, recent_protect=2, sim_metric="scaled_dot_product")),
    "hy_decode_bf16_cosine_b2": lambda M, S: case_hy_decode(
        M, "hyd2", 200, "bf16", 2, 1, 128, 10, 16, 1, 9, 0,
        dict(tile_size=(4, 8, 4), topk_ratio=0.175, recent_protect=4, sim_metric="cosine")),
    "hy_prefill_bf16_text": lambda M, S: case_hy_prefill(
        M, S, "hyp", 300, "bf16", 1, 2, 128, 12, 16, 8, 7,
        dict(tile_size=(4, 8, 4), topk_ratio=0.3, sim_metric="scaled_dot_product")),
    "mg_bidir_bf16": lambda M, S: case_mg(
        M, "mg", 400, "bf16", 1, 2, 128, 10, 20, 6, 0,
        dict(tile_size=(4, 4, 8), topk_ratio=0.3, sim_metric="cosine")),
    "mg_bidir_bf16_text": lambda M, S: case_mg(
        M, "mgt", 500, "bf16", 1, 1, 128, 8, 16, 4, 130,
        dict(tile_size=(4, 4, 8), topk_ratio=0.3, sim_metric="cosine")),
    "sel_decode_ties_bf16": lambda M, S: case_selection(
        M, "st", 600, "bf16", "decode", 1, 3, 128, (1, 4, 4), (8, 4, 4), 0,
        dict(tile_size=(1, 8, 16), topk_ratio=0.25, recent_protect=2, sim_metric="dot"), quant=4),
    "sel_bidir_ties_bf16": lambda M, S: case_selection(
        M, "sb", 700, "bf16", "bidir_mg", 1, 2, 128, (5, 4, 4), (5, 4, 4), 130,
        dict(tile_size=(4, 4, 8), topk_ratio=0.3, sim_metric="cosine"), quant=2),
    "sel_decode_small_fp32": lambda M, S: case_selection(
        M, "ss", 800, "fp32", "decode", 1, 2, 64, (1, 1, 2), (2, 1, 2), 3,
        dict(tile_size=(2, 4, 8), topk_ratio=0.1, recent_protect=9, sim_metric="cosine")),
    "sel_bidir_small_bf16": lambda M, S: case_selection(
        M, "sm", 900, "bf16", "bidir_hy", 2, 1, 64, (1, 2, 3), (1, 2, 3), 0,
        dict(tile_size=(4, 4, 8), topk_ratio=0.3, sim_metric="scaled_dot_product")),
}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref-root", default=os.environ.get("LI_REFERENCE_ROOT"),
                    help="root of the reference checkout (required; or set LI_REFERENCE_ROOT)")
    ap.add_argument("--only", nargs="*")
    args = ap.parse_args()
    if not args.ref_root:
        ap.error("--ref-root (or LI_REFERENCE_ROOT) must name the reference checkout")
    torch.manual_seed(0)
    mods, state = _load_reference(args.ref_root)
    for name, fn in CASES.items():
        if args.only and name not in args.only:
            continue
        res = fn(mods, state)
        meta = res.pop("meta")
        kind = res.pop("kind")
        sha = res.pop("inputs_sha")
        arrays = {}
        for k, v in res.items():
            a = np.asarray(v)
            if a.dtype == np.float32 and meta["dtype"] == "bf16" and k not in ("out_masked", "rank_scores"):
                # bf16-valued: store the bit patterns (exact, half the size).
                arrays[k + "__bf16"] = li_oracle.bf16_bits(a)
            else:
                arrays[k] = a
        np.savez_compressed(os.path.join(HERE, name + ".npz"),
                            meta=json.dumps(dict(meta, kind=kind, inputs_sha=sha)), **arrays)
        print(f"{name}: {', '.join(f'{k}{list(np.asarray(v).shape)}' for k, v in arrays.items())}")


if __name__ == "__main__":
    main()
