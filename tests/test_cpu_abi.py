"""CPU-only checks of the C ABI library and the host-side logic (no GPU calls)."""

import ctypes
import os
import re

import numpy as np
import pytest

from light_interaction_project_b200 import _lib as L
from light_interaction_project_b200 import build_lib
from light_interaction_project_b200 import kernels as K
from oracle import li_oracle as O

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include", "li_b200.h")


@pytest.fixture(scope="module")
def lib():
    build_lib.build()
    return L.load()


def declared_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"^(?:li_status|const char\*|uint64_t)\s+(li_\w+)\s*\(", text, flags=re.M)))


def test_header_declares_every_bound_symbol():
    assert declared_symbols() == sorted(L.SIGNATURES)


def test_library_exports_every_declared_symbol(lib):
    for name in declared_symbols():
        assert hasattr(lib, name), name
    assert lib.li_version().decode().startswith("li_b200")


@pytest.mark.parametrize("nk", [0, 1, 5, 63, 64, 192, 256, 280, 952, 1024])
@pytest.mark.parametrize("ratio", [0.0, 0.1, 0.175, 0.25, 0.3, 0.5, 1.0])
@pytest.mark.parametrize("rp", [0, 1, 2, 4, 9])
def test_decode_budget_matches_reference_formula(lib, nk, ratio, rp):
    tile, gq = (4, 8, 4), (1, 4, 4)
    p = K.select_params(L.SELECT_DECODE, "cosine", tile, gq, (8, 4, 4), 5, rp, ratio)
    ntxt, k = K.select_budget(p, 16, nk)
    n_prot, ref_k = O.decode_budget(nk, tile, gq, dict(recent_protect=rp, topk_ratio=ratio))
    assert (ntxt, k) == (1, ref_k)


@pytest.mark.parametrize("nk", [0, 1, 6, 7, 8, 23, 280, 1120])
@pytest.mark.parametrize("ratio", [0.0, 0.1, 0.25, 0.3, 0.5, 1.0])
def test_bidir_budget_matches_reference_formula(lib, nk, ratio):
    p = K.select_params(L.SELECT_BIDIR, "cosine", (4, 4, 8), (1, 1, 1), (1, 1, 1), 130, 0, ratio)
    ntxt, k = K.select_budget(p, nk, nk)
    assert (ntxt, k) == (2, O.prefill_budget(nk, ratio))


def test_entry_points_validate_before_launch(lib):
    """Null or inconsistent arguments come back as status codes; nothing launches."""
    assert lib.li_tile_pool(None, None, None, L.grid3d(1, 1, 1, (1, 1, 1)), None, None, 0, None, 0, None) == L.LI_ERR_INVALID_ARG
    assert "src0" in L.last_error()
    v = L.View4()
    v.data = 16
    for i, (s, st) in enumerate(zip((1, 1, 64, 128), (8192, 8192, 128, 1))):
        v.shape[i], v.stride[i] = s, st
    v.dtype = L.DTYPE_BF16
    bad_grid = L.grid3d(1, 8, 8, (1, 8, 0))
    assert lib.li_tile_pool(ctypes.byref(v), None, None, bad_grid, None, None, 0, None, 0, None) == L.LI_ERR_SHAPE
    v.dtype = 7
    assert lib.li_tile_pool(ctypes.byref(v), None, None, L.grid3d(1, 8, 8, (1, 8, 8)), None, None, 0, None, 0,
                            None) == L.LI_ERR_INVALID_ARG
    # Attention: fp32 operands are not built (the Python layer casts them).
    v.dtype = L.DTYPE_FP32
    iv = L.IndexView()
    st = lib.li_sparse_attn_tiled(ctypes.byref(v), ctypes.byref(v), ctypes.byref(v), ctypes.byref(iv), 128, 1.0,
                                  ctypes.byref(v), None, None, None, 0, None)
    assert st == L.LI_ERR_UNSUPPORTED
    v.dtype = L.DTYPE_BF16
    st = lib.li_sparse_attn_tiled(ctypes.byref(v), ctypes.byref(v), ctypes.byref(v), ctypes.byref(iv), 96, 1.0,
                                  ctypes.byref(v), None, None, None, 0, None)
    assert st == L.LI_ERR_UNSUPPORTED
    with pytest.raises(NotImplementedError):
        L.check(st, "attn")


def test_selection_scratch_sizes_never_overflow(lib):
    """The selection's key-scratch size saturates instead of wrapping, negative
    shapes are refused, and the no-allocation entry point refuses a negative pool
    shape before touching the device."""
    nbytes = ctypes.c_int64()
    assert lib.li_select_workspace_bytes(1, 24, 56, 952, ctypes.byref(nbytes)) == L.LI_OK
    assert nbytes.value == 24 * 56 * 952 * 4
    assert lib.li_select_workspace_bytes(1 << 40, 1 << 40, 1, 1, ctypes.byref(nbytes)) == L.LI_OK
    assert nbytes.value == 2 ** 63 - 1
    assert lib.li_select_workspace_bytes(-1, 24, 56, 952, ctypes.byref(nbytes)) == L.LI_ERR_SHAPE
    q = L.View4()
    q.data = 256
    for i, (sh, st) in enumerate(zip((-1, 1, 4, 128), (512, 512, 128, 1))):
        q.shape[i], q.stride[i] = sh, st
    q.dtype = L.DTYPE_BF16
    p = K.select_params(L.SELECT_DECODE, "dot", (1, 8, 16), (1, 2, 2), (1, 2, 2), 0, 0, 1.0)
    iv = L.IndexView()
    st = lib.li_select_blocks_static(ctypes.byref(q), ctypes.byref(q), ctypes.byref(p), None, ctypes.byref(iv),
                                     None, None)
    assert st == L.LI_ERR_SHAPE and "non-negative" in L.last_error()


def test_split_plan_workspace(lib):
    """Tail split: only the tiles of a mostly idle last wave (148 SMs, one CTA
    each) are cut into list pieces; the workspace holds exactly their partials."""
    nbytes = ctypes.c_int64()
    unit = 128 * 130 * 4   # one fp32 partial tile of D=128: O, row max, row sum
    assert lib.li_sparse_attn_workspace_bytes(1, 24, 56, 238, 128, 128, ctypes.byref(nbytes)) == 0
    assert nbytes.value == 12 * 12 * unit        # 1344 tiles = 9 waves + 12: each of the 12 in 12 pieces
    assert lib.li_sparse_attn_workspace_bytes(1, 3, 56, 238, 128, 128, ctypes.byref(nbytes)) == 0
    assert nbytes.value == 20 * 7 * unit         # 168 tiles = 1 wave + 20: 7 pieces each
    assert lib.li_sparse_attn_workspace_bytes(1, 16, 64, 256, 128, 128, ctypes.byref(nbytes)) == 0
    assert nbytes.value == 0                     # 1024 tiles = 6 waves + 136: last wave nearly full
    assert lib.li_sparse_attn_workspace_bytes(1, 148, 1, 100, 128, 128, ctypes.byref(nbytes)) == 0
    assert nbytes.value == 0                     # whole waves
    assert lib.li_sparse_attn_workspace_bytes(1, 3, 56, 8, 128, 128, ctypes.byref(nbytes)) == 0
    assert nbytes.value == 0                     # too few blocks per row to split


def test_rank_blocks_rejects_k_out_of_range(lib):
    v = L.View4()
    v.data = 256
    for i, (s, st) in enumerate(zip((1, 1, 4, 10), (40, 40, 10, 1))):
        v.shape[i], v.stride[i] = s, st
    v.dtype = L.DTYPE_FP32
    iv = L.IndexView()
    assert lib.li_rank_blocks(ctypes.byref(v), L.DTYPE_BF16, 11, 0, 128, ctypes.byref(iv), None) == L.LI_ERR_OUT_OF_BOUNDS


def test_tensor_wrappers_refuse_cpu_tensors():
    import torch
    with pytest.raises(ValueError, match="CUDA"):
        L.view4(torch.zeros(1, 1, 1, 8), "x")


_STRUCTS = {"li_view4": L.View4, "li_view5": L.View5, "li_index_view": L.IndexView, "li_grid3d": L.Grid3d,
            "li_select_params": L.SelectParams, "li_a2a_desc": L.A2ADesc}


def test_ctypes_structs_match_header_layout(tmp_path):
    """Field order, offsets and sizes of every C-ABI struct, as gcc lays them out
    from the header, equal the ctypes mirrors."""
    import shutil
    import subprocess
    if shutil.which("gcc") is None:
        pytest.skip("gcc not available")
    lines = ["#include <stdio.h>", "#include <stddef.h>", f'#include "{HEADER}"', "int main(void) {"]
    for cname, cls in _STRUCTS.items():
        lines.append(f'printf("{cname} size %zu\\n", sizeof({cname}));')
        for fname, _ in cls._fields_:
            lines.append(f'printf("{cname} {fname} %zu %zu\\n", offsetof({cname}, {fname}), '
                         f'sizeof((({cname}*)0)->{fname}));')
    lines += ["return 0;", "}"]
    src, exe = tmp_path / "layout.c", tmp_path / "layout"
    src.write_text("\n".join(lines))
    subprocess.run(["gcc", "-std=c11", "-o", str(exe), str(src)], check=True, capture_output=True)
    out = subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout.split("\n")
    got = {}
    for row in out:
        parts = row.split()
        if len(parts) == 3:
            got[(parts[0], "__size__")] = int(parts[2])
        elif len(parts) == 4:
            got[(parts[0], parts[1])] = (int(parts[2]), int(parts[3]))
    for cname, cls in _STRUCTS.items():
        assert got[(cname, "__size__")] == ctypes.sizeof(cls), cname
        for fname, _ in cls._fields_:
            f = getattr(cls, fname)
            assert got[(cname, fname)] == (f.offset, f.size), f"{cname}.{fname}"
    # every header field is mirrored (no field missing from a ctypes struct)
    text = open(HEADER).read()
    for cname, cls in _STRUCTS.items():
        body = re.search(r"typedef struct " + cname + r" \{(.*?)\} " + cname + ";", text, flags=re.S).group(1)
        body = re.sub(r"/\*.*?\*/", "", body, flags=re.S)
        names = []
        for decl in body.split(";"):
            decl = decl.strip()
            if not decl:
                continue
            for part in decl.split(","):
                names.append(re.sub(r"\[.*?\]", "", part).replace("*", " ").split()[-1])
        assert names == [n for n, _ in cls._fields_], cname
