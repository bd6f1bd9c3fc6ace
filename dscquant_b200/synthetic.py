"""Seeded synthetic inputs with the distributions of the W4A4 benchmark configs.

Activations ~ N(0, 1) with 1% of the K input channels (seeded choice) scaled
x20 as outliers; weights ~ N(0, 0.02). Values are produced in float32 by
numpy's PCG64 (bit-identical on every machine) and rounded to bfloat16 with
round-to-nearest-even, so tests, fixtures and benchmarks regenerate exactly
the same tensors from (shape, seed).
"""
from __future__ import annotations

import numpy as np


def _to_bf16_bits(x: np.ndarray) -> np.ndarray:
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def activations_bf16(M: int, K: int, seed: int = 0, outlier_frac: float = 0.01, outlier_scale: float = 20.0):
    """[M, K] bf16 bit patterns (uint16)."""
    rng = np.random.Generator(np.random.PCG64(seed))
    x = rng.standard_normal((M, K), dtype=np.float32)
    n_out = max(1, int(K * outlier_frac))
    cols = np.random.Generator(np.random.PCG64(seed + 7919)).permutation(K)[:n_out]
    x[:, cols] *= np.float32(outlier_scale)
    return _to_bf16_bits(x)


def weights_bf16(N: int, K: int, seed: int = 1, std: float = 0.02):
    """[N, K] bf16 bit patterns (uint16)."""
    rng = np.random.Generator(np.random.PCG64(seed))
    w = rng.standard_normal((N, K), dtype=np.float32) * np.float32(std)
    return _to_bf16_bits(w)


def to_torch_bf16(bits: np.ndarray, device=None):
    import torch

    t = torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16)
    return t.to(device) if device is not None else t
