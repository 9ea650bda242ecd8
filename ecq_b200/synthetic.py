"""Seeded synthetic inputs for the decode + dequant + GEMV workloads.

The reference measures on no public dataset; its benchmark shapes are the
Llama-7B / 70B layer shapes with 4-bit symbols drawn from a discrete Laplace
centred at 8. These generators make those inputs deterministically:

* symbols: ``rng.choice(16, p = p_b)`` with ``p_b(k) ∝ exp(-|k-8| / b)``
  (seed 0), row-major [M, K];
* scales:  fp16 ``U(0.01, 0.03)`` of shape [M, ceil(K/g)] (seed 1), zero-point 8;
* x:       fp16 ``N(0, 1)`` of shape [B, K] (seed 2);
* Student-t weights for a full-model step: fp16 ``t(4) * 0.02`` quantised
  symmetrically per group (absmax/7, zero-point 8).
"""
from __future__ import annotations

import numpy as np


def laplace_probs(b: float) -> np.ndarray:
    k = np.arange(16, dtype=np.float64)
    p = np.exp(-np.abs(k - 8.0) / float(b))
    return p / p.sum()


def entropy_bits(p) -> float:
    p = np.asarray(p, dtype=np.float64)
    p = p[p > 0]
    return float(-(p * np.log2(p)).sum())


def laplace_symbols(M: int, K: int, b: float = 0.5, seed: int = 0) -> np.ndarray:
    rng = np.random.default_rng(seed)
    return rng.choice(16, size=M * K, p=laplace_probs(b)).astype(np.uint8).reshape(M, K)


def group_scales(M: int, K: int, group_size: int, seed: int = 1) -> np.ndarray:
    rng = np.random.default_rng(seed)
    ng = (K + group_size - 1) // group_size
    return rng.uniform(0.01, 0.03, (M, ng)).astype(np.float16)


def activations(B: int, K: int, seed: int = 2) -> np.ndarray:
    rng = np.random.default_rng(seed)
    return rng.standard_normal((B, K)).astype(np.float16)


def quantize_symmetric_groups(w: np.ndarray, group_size: int = 128):
    """Symmetric per-group 4-bit quantiser: scale = absmax/7, q = clip(round(w/scale)+8,
    0, 15). Returns (symbols uint8 [M,K], scales fp16 [M, K/g])."""
    w = np.asarray(w, dtype=np.float32)
    M, K = w.shape
    assert K % group_size == 0, "K must be a multiple of the group size"
    wg = w.reshape(M, K // group_size, group_size)
    amax = np.abs(wg).max(axis=2)
    scale = (amax / 7.0).astype(np.float16)
    sc32 = scale.astype(np.float32)
    safe = np.where(sc32 == 0, 1.0, sc32)
    q = np.clip(np.rint(wg / safe[:, :, None]) + 8, 0, 15).astype(np.uint8)
    return q.reshape(M, K), scale


def student_t_weights(M: int, K: int, seed: int) -> np.ndarray:
    rng = np.random.default_rng(seed)
    return (rng.standard_t(4, (M, K)) * 0.02).astype(np.float16)
