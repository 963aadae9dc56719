"""TurboQuant constants (get_turbo_constants, src/foveated_kv/turbo_constants.py:29-100).

Pi: QR of a RandomState(42) Gaussian (d, d) float32 matrix, columns sign-fixed
so diag(R) > 0.  S: RandomState(137) Gaussian / sqrt(d).  Centroids and
decision boundaries: 200 Lloyd-Max iterations for N(0, 1/d) at 2 bits.
Computed once per (d, device) on the host (as the reference does) and kept
resident on the device as float32.
"""

from __future__ import annotations

from dataclasses import dataclass
from functools import lru_cache

import numpy as np


@dataclass(frozen=True)
class TurboConstants:
    Pi: "object"          # (D, D) float32 torch tensor
    S: "object"           # (D, D) float32
    centroids: "object"   # (4,) float32
    boundaries: "object"  # (3,) float32


def rotation_matrix(d: int, seed: int = 42) -> np.ndarray:
    rng = np.random.RandomState(seed)
    h = rng.randn(d, d).astype(np.float32)
    q, r = np.linalg.qr(h)
    sg = np.sign(np.diag(r))
    sg[sg == 0] = 1
    return (q * sg[np.newaxis, :]).astype(np.float32)


def qjl_matrix(d: int, seed: int = 137) -> np.ndarray:
    rng = np.random.RandomState(seed)
    return (rng.randn(d, d).astype(np.float32) / np.sqrt(d)).astype(np.float32)


def lloyd_max(d: int, bits: int = 2, n_iters: int = 200):
    from scipy.stats import norm
    n = 2 ** bits
    sigma = 1.0 / np.sqrt(d)
    b = norm.ppf(np.linspace(0, 1, n + 1)[1:-1], scale=sigma)
    c = np.zeros(n)
    for _ in range(n_iters):
        ext = np.concatenate([[-np.inf], b, [np.inf]])
        c = np.zeros(n)
        for i in range(n):
            lo, hi = ext[i], ext[i + 1]
            prob = norm.cdf(hi, scale=sigma) - norm.cdf(lo, scale=sigma)
            if prob > 1e-15:
                c[i] = sigma ** 2 * (norm.pdf(lo, scale=sigma) - norm.pdf(hi, scale=sigma)) / prob
            else:
                c[i] = (lo + hi) / 2 if np.isfinite(lo + hi) else 0
        b = (c[:-1] + c[1:]) / 2
    return c.astype(np.float32), b.astype(np.float32)


@lru_cache(maxsize=4)
def host_constants(d: int, pi_seed: int = 42, s_seed: int = 137):
    c, b = lloyd_max(d)
    return rotation_matrix(d, pi_seed), qjl_matrix(d, s_seed), c, b


@lru_cache(maxsize=8)
def get_turbo_constants(d: int, device: str = "cuda") -> TurboConstants:
    import torch
    pi, s, c, b = host_constants(d)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(device)
    return TurboConstants(Pi=t(pi), S=t(s), centroids=t(c), boundaries=t(b))
