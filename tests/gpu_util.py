"""Helpers shared by the GPU parity tests."""

import numpy as np
import torch

from oracle.inputs import det_normal_like

TORCH_DT = {"bf16": torch.bfloat16, "fp16": torch.float16, "fp32": torch.float32}


def dev():
    return torch.device("cuda", 0)


def to_gpu(a: np.ndarray, dtype: str) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(dev()).to(TORCH_DT[dtype])


def to_np(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().cpu().numpy()


def rand(shape, seed, dtype, scale=1.0):
    """Seeded input (bit-reproducible) rounded to ``dtype``; returns (numpy, gpu)."""
    from oracle.li_oracle import round_to
    if dtype == "fp16":
        a = det_normal_like(shape, seed, "fp32", scale).astype(np.float16).astype(np.float32)
    else:
        a = det_normal_like(shape, seed, dtype, scale)
    return a, to_gpu(a, dtype)


def assert_close_bf16(got: np.ndarray, ref: np.ndarray, max_abs=2e-2, mean_abs=2e-3, what=""):
    d = np.abs(got.astype(np.float64) - ref.astype(np.float64))
    assert np.isfinite(got).all(), f"{what}: non-finite output"
    assert d.max() <= max_abs and d.mean() <= mean_abs, f"{what}: max-abs {d.max():.3e} mean-abs {d.mean():.3e}"
