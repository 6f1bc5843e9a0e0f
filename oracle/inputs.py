"""Bit-reproducible synthetic inputs for the golden fixtures (test infrastructure).

The fixtures under ``tests/golden`` store seeds, not input tensors. Inputs are
rebuilt here with integer arithmetic (splitmix64) and exact IEEE float64 adds
and multiplies (Irwin-Hall sum of four uniforms, scaled to unit variance).
No libm call is involved, so every machine and numpy version produces the
same bits. Values are approximately N(0, 1).
"""

import numpy as np

_M64 = np.uint64(0xFFFFFFFFFFFFFFFF)


def _splitmix64(state: np.ndarray) -> np.ndarray:
    z = state
    z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
    z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
    return z ^ (z >> np.uint64(31))


def det_uniform(n: int, seed: int, stream: int = 0) -> np.ndarray:
    """``n`` float64 values in [0, 1) from counter-mode splitmix64."""
    with np.errstate(over="ignore"):
        base = np.uint64((seed * 0x9E3779B97F4A7C15 + stream * 0xD1B54A32D192ED03) & 0xFFFFFFFFFFFFFFFF)
        ctr = np.arange(n, dtype=np.uint64) * np.uint64(0x9E3779B97F4A7C15) + base
        bits = _splitmix64(ctr)
    return (bits >> np.uint64(11)).astype(np.float64) * (1.0 / 9007199254740992.0)


def det_normal(shape, seed: int, scale: float = 1.0) -> np.ndarray:
    """Approximately N(0, scale^2) float64 array, identical on every machine."""
    n = int(np.prod(shape)) if len(shape) else 1
    acc = np.zeros(n, dtype=np.float64)
    for s in range(4):
        acc = acc + det_uniform(n, seed, s)
    # Irwin-Hall(4): mean 2, variance 1/3.
    out = (acc - 2.0) * 1.7320508075688772 * scale
    return out.reshape(shape)


def det_normal_like(shape, seed: int, dtype: str, scale: float = 1.0) -> np.ndarray:
    """``det_normal`` rounded to ``dtype`` ('bf16' or 'fp32'); returned as float32."""
    from .li_oracle import round_to
    return round_to(det_normal(shape, seed, scale).astype(np.float32), dtype)
