"""Seeded synthetic inputs for the parity tests and the benchmark.

Values come from PCG64's raw 64-bit stream (whose output numpy keeps stable
across releases) through integer arithmetic and one IEEE rounding, so the
same seed gives the same float32 bits on every machine.  ``normalish`` sums
four 24-bit uniforms (Irwin-Hall) and rescales to mean 0, variance 1: a
bounded stand-in for N(0, 1) with the same first two moments.
"""
from __future__ import annotations

import numpy as np


def _raw(seed: int, n: int) -> np.ndarray:
    return np.random.PCG64(seed).random_raw(n)


def normalish(seed: int, shape, scale: float = 1.0) -> np.ndarray:
    n = int(np.prod(shape))
    raw = _raw(seed, 4 * n).reshape(4, n)
    s = (raw >> np.uint64(40)).astype(np.int64).sum(axis=0)
    x = (s.astype(np.float64) / float(1 << 24) - 2.0) * np.sqrt(3.0) * scale
    return x.astype(np.float32).reshape(shape)


def uniform_int(seed: int, shape, lo: int, hi: int) -> np.ndarray:
    """Integers uniform in [lo, hi] (inclusive)."""
    n = int(np.prod(shape))
    raw = _raw(seed, n)
    return (lo + (raw % np.uint64(hi - lo + 1)).astype(np.int64)).reshape(shape)


def outlier_rows(seed: int, n_rows: int, frac: float) -> np.ndarray:
    """Distinct row indices (sorted), round(frac * n_rows) of them."""
    m = int(round(frac * n_rows))
    raw = _raw(seed, n_rows)
    return np.sort(np.argsort(raw, kind="stable")[:m])


def bf16_round(x: np.ndarray) -> np.ndarray:
    """float32 -> nearest bf16 value (ties to even), returned as float32."""
    u = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
    return r.astype(np.uint32).view(np.float32)


def bf16_bits(x: np.ndarray) -> np.ndarray:
    """float32 values that are exact bf16 -> uint16 bit patterns."""
    return (np.ascontiguousarray(x, np.float32).view(np.uint32) >> 16).astype(np.uint16)


def stage1_inputs(seed: int, H: int, HK: int, D: int, len_q: int, len_k: int):
    Q = normalish(seed, (H, len_q, D))
    K = normalish(seed + 1, (HK, len_k, D))
    return Q, K


def stage2_inputs(seed: int, H: int, HK: int, D: int, L: int, outlier_frac: float = 0.01,
                  outlier_scale: float = 8.0, bf16: bool = True):
    q = normalish(seed, (H, D))
    K = normalish(seed + 1, (HK, L, D))
    V = normalish(seed + 2, (HK, L, D))
    if outlier_frac > 0:
        for h in range(HK):
            rows = outlier_rows(seed + 100 + h, L, outlier_frac)
            K[h, rows, :] *= np.float32(outlier_scale)
    if bf16:
        q, K, V = bf16_round(q), bf16_round(K), bf16_round(V)
    return q, K, V


def q8_0_inputs(seed: int, lead_shape, D: int):
    """q8_0 rows: int8 uniform in [-127, 127], fp16 scales |N(0, 0.02)|.
    Returns (packed uint8 [..., D/32*34], exact float32 dequantisation)."""
    nb = D // 32
    qs = uniform_int(seed, tuple(lead_shape) + (nb, 32), -127, 127).astype(np.int8)
    sc = np.abs(normalish(seed + 7, tuple(lead_shape) + (nb,), 0.02)).astype(np.float16)
    packed = np.zeros(tuple(lead_shape) + (nb, 34), np.uint8)
    packed[..., 0:2] = sc.view(np.uint8).reshape(tuple(lead_shape) + (nb, 2))
    packed[..., 2:] = qs.view(np.uint8)
    deq = (sc.astype(np.float32)[..., None] * qs.astype(np.float32)).reshape(tuple(lead_shape) + (D,))
    return packed.reshape(tuple(lead_shape) + (nb * 34,)), deq.astype(np.float32)
