"""Seeded synthetic inputs for every configuration (there is no dataset on
this path: the reference's benchmarks run on random weights and vectors).

One recipe, implemented twice with the same arithmetic: ``fill_normal``
(numpy, host) and ``xpu_fill_normal_f32_dev`` (CUDA, device).  Element i:

    h(lane) = mix64(seed * 0x9E3779B97F4A7C15 + (3*i + lane + 1) * 0xD1B54A32D192ED03)
    u1 = ((h(0) >> 11) + 1) * 2^-53          in (0, 1]
    u2 = (h(1) >> 11) * 2^-53                in [0, 1)
    z  = sqrt(-2 ln u1) * cos(2 pi u2)       (Box-Muller, f64)
    v  = mean + std * z;  v *= outlier_mul if (h(2) >> 11) * 2^-53 < outlier_frac
    out[i] = float32(v)

mix64 is splitmix64's output function.  Host and device agree exactly except
where f64 `log`/`cos` differ in the last place between libm and CUDA, which
can move a result by one f32 ulp.
"""
from __future__ import annotations

import numpy as np

_M1 = np.uint64(0xBF58476D1CE4E5B9)
_M2 = np.uint64(0x94D049BB133111EB)
_G = np.uint64(0x9E3779B97F4A7C15)
_S = np.uint64(0xD1B54A32D192ED03)


def _mix64(z: np.ndarray) -> np.ndarray:
    z = (z ^ (z >> np.uint64(30))) * _M1
    z = (z ^ (z >> np.uint64(27))) * _M2
    return z ^ (z >> np.uint64(31))


def _hash3(seed: int, i: np.ndarray, lane: int) -> np.ndarray:
    with np.errstate(over="ignore"):
        base = np.uint64(seed) * _G
        return _mix64(base + (np.uint64(3) * i + np.uint64(lane + 1)) * _S)


def fill_normal(n: int, seed: int, mean: float = 0.0, std: float = 1.0, outlier_frac: float = 0.0,
                outlier_mul: float = 1.0, start: int = 0) -> np.ndarray:
    """Elements [start, start + n) of the seeded stream, as float32."""
    i = np.arange(start, start + n, dtype=np.uint64)
    inv53 = 1.0 / 9007199254740992.0
    with np.errstate(over="ignore"):
        u1 = ((_hash3(seed, i, 0) >> np.uint64(11)) + np.uint64(1)).astype(np.float64) * inv53
        u2 = (_hash3(seed, i, 1) >> np.uint64(11)).astype(np.float64) * inv53
    z = np.sqrt(-2.0 * np.log(u1)) * np.cos(6.283185307179586 * u2)
    v = mean + std * z
    if outlier_frac > 0.0:
        u3 = (_hash3(seed, i, 2) >> np.uint64(11)).astype(np.float64) * inv53
        v = np.where(u3 < outlier_frac, v * outlier_mul, v)
    return v.astype(np.float32)


def tensor_seed(base_seed: int, index: int) -> int:
    """Seed of the index-th tensor of a model built from `base_seed`."""
    return (int(base_seed) * 1_000_003 + int(index)) & 0xFFFFFFFFFFFFFFFF


# ---- the reference's own deterministic test inputs (ops/matvec/*.wgsl.test.ts)

def code_wave(n: int, k: float, phase: float = 0.0) -> np.ndarray:
    """ops/matvec/q8.wgsl.test.ts:23-24: Math.round(Math.sin(i*k + phase) * 100)."""
    v = np.sin(np.arange(n, dtype=np.float64) * k + phase) * 100.0
    f = np.floor(v)
    return (f + ((v - f) >= 0.5)).astype(np.int32)


def wave(n: int, k: float, phase: float = 0.0) -> np.ndarray:
    """ops/matvec/q8.wgsl.test.ts:25-26: Math.sin(i*k + phase) * 1.5, as f32."""
    return (np.sin(np.arange(n, dtype=np.float64) * k + phase) * 1.5).astype(np.float32)


def scale_wave(n: int, phase: float = 0.007) -> np.ndarray:
    """ops/matvec/q8.wgsl.test.ts:28: 0.02 * (i + 1) + 0.007, as f32."""
    return (0.02 * (np.arange(n, dtype=np.float64) + 1.0) + phase).astype(np.float32)


def residual_wave(n: int) -> np.ndarray:
    """ops/matvec/q8_residual.wgsl.test.ts:16: Math.cos(i*0.29 + 2.1) * 5."""
    return (np.cos(np.arange(n, dtype=np.float64) * 0.29 + 2.1) * 5.0).astype(np.float32)
