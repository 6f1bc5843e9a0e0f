"""Loading helpers for the golden fixtures in ``tests/golden`` (test support)."""

import glob
import json
import os

import numpy as np

GOLDEN_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def list_cases(prefix=""):
    return sorted(os.path.basename(p)[:-4] for p in glob.glob(os.path.join(GOLDEN_DIR, prefix + "*.npz")))


def load_case(name):
    z = np.load(os.path.join(GOLDEN_DIR, name + ".npz"))
    meta = json.loads(str(z["meta"]))
    out = {}
    for k in z.files:
        if k == "meta":
            continue
        if k.endswith("__bf16"):
            out[k[:-6]] = (z[k].astype(np.uint32) << 16).view(np.float32)
        else:
            out[k] = z[k]
    return meta, out


def rebuild_inputs(meta):
    """Rebuild the seeded inputs of a fixture (bit-identical to generation)."""
    from oracle.inputs import det_normal_like
    s, dt = meta["seed"], meta["dtype"]
    B, H, D = meta["B"], meta["H"], meta["D"]
    kind = meta["kind"]
    if kind.startswith("selection"):
        raise ValueError("selection fixtures store their pools")
    HW = meta["LH"] * meta["LW"]
    if kind == "mg":
        tl, F = meta["text_len"], meta["Fq"]
        return dict(q=det_normal_like((B, H, F * HW, D), s, dt),
                    k=det_normal_like((B, H, tl + F * HW, D), s + 3, dt),
                    v=det_normal_like((B, H, tl + F * HW, D), s + 4, dt))
    tl = meta["text_len"]
    return dict(q=det_normal_like((B, H, meta["Fq"] * HW, D), s, dt),
                k_txt=det_normal_like((B, H, tl, D), s + 1, dt),
                v_txt=det_normal_like((B, H, tl, D), s + 2, dt),
                k_vis=det_normal_like((B, H, meta["Fk"] * HW, D), s + 3, dt),
                v_vis=det_normal_like((B, H, meta["Fk"] * HW, D), s + 4, dt))


def input_checksum(meta, inputs):
    import hashlib
    h = hashlib.sha256()
    order = ("q", "k", "v") if meta["kind"] == "mg" else ("q", "k_txt", "v_txt", "k_vis", "v_vis")
    for k in order:
        h.update(np.ascontiguousarray(inputs[k], np.float32).tobytes())
    return h.hexdigest()


def tie_explained(ref_idx, got_idx, scores, dtype, ntxt):
    """True when two ascending index rows select score multisets that are equal
    and every differing index carries the k-th (boundary) score — i.e. they differ
    only in which of several exactly-equal scores was kept."""
    from oracle.li_oracle import radix_key
    a = set(int(x) - ntxt for x in ref_idx[ntxt:])
    b = set(int(x) - ntxt for x in got_idx[ntxt:])
    if a == b:
        return True
    keys = radix_key(np.asarray(scores, np.float32), dtype)
    ka = sorted(int(keys[i]) for i in a)
    kb = sorted(int(keys[i]) for i in b)
    if ka != kb:
        return False
    kth = ka[0]
    return all(int(keys[i]) == kth for i in a.symmetric_difference(b))
