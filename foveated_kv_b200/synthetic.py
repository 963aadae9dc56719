"""Seeded synthetic decode workloads (the reference benchmarks on synthetic
N(0,1) fp16 K/V/q only: benchmarks/benchmark_mlx.py:77-84,135-204).

K, V, q ~ N(0, 1) in fp16; per KV head, 4 K channels picked by a seeded
permutation are scaled x8 (outlier channels).  Two generators with the same
distribution: a NumPy one (bit-stable across machines, used for parity
fixtures) and a torch one that draws directly on the device (used for
full-size benchmarks, where host generation would dominate).
"""

from __future__ import annotations

import numpy as np

N_OUTLIER_CHANNELS = 4
OUTLIER_SCALE = 8.0


def numpy_workload(seed: int, B: int, Hk: int, Hq: int, S: int, D: int, n_dec: int = 0):
    """Returns dict of fp16 arrays: k, v (B,Hk,S,D), q (B,Hq,D), q_obs (B,Hq,D),
    dec_k, dec_v (B,Hk,n_dec,D)."""
    rs = np.random.RandomState(seed)
    k = rs.standard_normal((B, Hk, S, D)).astype(np.float32)
    v = rs.standard_normal((B, Hk, S, D)).astype(np.float32)
    for h in range(Hk):
        ch = rs.permutation(D)[:N_OUTLIER_CHANNELS]
        k[:, h, :, ch] *= OUTLIER_SCALE
    q = rs.standard_normal((B, Hq, D)).astype(np.float32)
    q_obs = rs.standard_normal((B, Hq, D)).astype(np.float32)
    dk = rs.standard_normal((B, Hk, n_dec, D)).astype(np.float32)
    dv = rs.standard_normal((B, Hk, n_dec, D)).astype(np.float32)
    f16 = lambda a: a.astype(np.float16)
    return {"k": f16(k), "v": f16(v), "q": f16(q), "q_obs": f16(q_obs),
            "dec_k": f16(dk), "dec_v": f16(dv)}


def torch_workload(seed: int, B: int, Hk: int, Hq: int, S: int, D: int, n_dec: int = 0,
                   device="cuda"):
    """Same distribution as ``numpy_workload``, drawn on ``device`` with a
    seeded torch generator (values differ from the NumPy stream)."""
    import torch
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    k = torch.randn((B, Hk, S, D), generator=g, device=device, dtype=torch.float16)
    v = torch.randn((B, Hk, S, D), generator=g, device=device, dtype=torch.float16)
    gc = torch.Generator()
    gc.manual_seed(seed)
    for h in range(Hk):
        ch = torch.randperm(D, generator=gc)[:N_OUTLIER_CHANNELS].to(device)
        k[:, h, :, ch] *= OUTLIER_SCALE
    q = torch.randn((B, Hq, D), generator=g, device=device, dtype=torch.float16)
    q_obs = torch.randn((B, Hq, D), generator=g, device=device, dtype=torch.float16)
    dk = torch.randn((B, Hk, n_dec, D), generator=g, device=device, dtype=torch.float16)
    dv = torch.randn((B, Hk, n_dec, D), generator=g, device=device, dtype=torch.float16)
    return {"k": k, "v": v, "q": q, "q_obs": q_obs, "dec_k": dk, "dec_v": dv}


# The benchmark configurations c0-c4 (shapes, tier settings, far-tier kind).
CONFIGS = {
    "c0": dict(B=1, Hq=14, Hk=2, D=64, S=1024, n_dec=16, near_pct=0.10, n_sinks=4,
               window_size=64, select="importance", v_group=32, compress_method="fp8"),
    "c1_1k": dict(B=1, Hq=32, Hk=32, D=128, S=1024, n_dec=0, near_pct=0.10, n_sinks=4,
                  window_size=128, select="recency", v_group=None, compress_method="fp8"),
    "c1_4k": dict(B=1, Hq=32, Hk=32, D=128, S=4096, n_dec=0, near_pct=0.10, n_sinks=4,
                  window_size=128, select="recency", v_group=None, compress_method="fp8"),
    "c1_8k": dict(B=1, Hq=32, Hk=32, D=128, S=8192, n_dec=0, near_pct=0.10, n_sinks=4,
                  window_size=128, select="recency", v_group=None, compress_method="fp8"),
    "c1_16k": dict(B=1, Hq=32, Hk=32, D=128, S=16384, n_dec=0, near_pct=0.10, n_sinks=4,
                   window_size=128, select="recency", v_group=None, compress_method="fp8"),
    "c2": dict(B=1, Hq=28, Hk=4, D=128, S=16384, n_dec=0, near_pct=0.10, n_sinks=4,
               window_size=32, select="recency", v_group=None, compress_method="turbo"),
    "c3": dict(B=64, Hq=32, Hk=8, D=128, S=32768, n_dec=0, near_pct=0.10, n_sinks=4,
               window_size=32, select="recency", v_group=None, compress_method="fp8"),
    "c4": dict(B=1, Hq=32, Hk=8, D=128, S=1 << 20, n_dec=0, near_pct=0.05, n_sinks=4,
               window_size=32, select="recency", v_group=None, compress_method="fp8"),
}


def spike_positions_np(seed: int, B: int, Hk: int, mid_start: int, F: int, frac: float = 0.01):
    """Seeded positions of the forced spikes: `max(1, int(F * frac))` far
    positions per (b, kv head) drawn uniformly from [mid_start, mid_start+F)."""
    n = max(1, int(F * frac))
    rs = np.random.RandomState(seed + 1)
    return mid_start + rs.randint(0, F, size=(B, Hk, n))


def inject_spikes_np(w: dict, tb: dict, seed: int, frac: float = 0.01):
    """Turn 1% of the far tokens of each (b, kv head) into spikes (config c3:
    "keys set to 3 sigma along q"): key = 3 sqrt(D) times the unit mean query
    of the GQA group, so their scores sit far above the lowest near score.
    In place on the NumPy workload ``w``; returns the positions."""
    k, q = w["k"], w["q"]
    B, Hk, S, D = k.shape
    G = q.shape[1] // Hk
    pos = spike_positions_np(seed, B, Hk, tb["mid_start"], tb["far_count"], frac)
    qm = q.astype(np.float32).reshape(B, Hk, G, D).mean(2)
    qm /= np.linalg.norm(qm, axis=-1, keepdims=True)
    val = (3.0 * D ** 0.5 * qm).astype(np.float16)
    for b in range(B):
        for h in range(Hk):
            k[b, h, pos[b, h]] = val[b, h]
    return pos


def inject_spikes_torch(w: dict, tb: dict, seed: int, frac: float = 0.01):
    """Device version of ``inject_spikes_np`` (same rule, torch generator)."""
    import torch
    k, q = w["k"], w["q"]
    B, Hk, S, D = k.shape
    G = q.shape[1] // Hk
    F = tb["far_count"]
    n = max(1, int(F * frac))
    g = torch.Generator(device=k.device)
    g.manual_seed(seed + 1)
    pos = tb["mid_start"] + torch.randint(0, F, (B, Hk, n), generator=g, device=k.device)
    qm = q.float().reshape(B, Hk, G, D).mean(2)
    qm = qm / qm.norm(dim=-1, keepdim=True)
    val = (3.0 * D ** 0.5 * qm).to(k.dtype)[:, :, None, :].expand(B, Hk, n, D)
    k.scatter_(2, pos[..., None].expand(B, Hk, n, D), val)
    return pos
