"""CPU restatement of the FoveatedKV decode hot path.

TEST INFRASTRUCTURE ONLY.  Nothing in the product (``foveated_kv_b200``)
imports this module; only ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` use it, and only
as the checker or the timed CPU arm.

Every function restates one piece of the reference's Python CPU path
(``src/foveated_kv/*.py`` of samfurr/foveated_kv 0.2.0) in NumPy, citing the
file:line it follows.  Where the reference is ambiguous or has no CPU code
(importance ranking, spike emission, turbo score-on-codes), the restatement
follows the reference's Metal *source* semantics or the written spec and says
so in the docstring.

Precision rules (kept identical in the CUDA kernels):
  * fp8 E4M3 and INT4 codes: integer bit arithmetic / IEEE fp32 ops
    (correctly rounded ``/``, round-half-even) -> bit-exact.
  * TurboQuant key codes and importance scores: fp64 accumulation, rounded to
    fp16 where the reference stores fp16.
  * Attention output: K/V dequantised to fp16 exactly as the reference does,
    then fp64 softmax attention (the reference uses MLX SDPA, which is not
    vendored; parity at tolerance level).
"""

from __future__ import annotations

import math
from typing import Optional

import numpy as np

# ---------------------------------------------------------------------------
# Tier boundaries -- mlx_foveated.py:128-169 (C++ copy foveated_compress.cpp:107-126)
# ---------------------------------------------------------------------------


def tier_boundaries(S: int, near_pct: float = 0.10, n_sinks: int = 4,
                    window_size: int = 32, promo_headroom_pct: float = 0.5,
                    promo_headroom_min: int = 8) -> dict:
    """Restates ``MLXTierConfig.tier_boundaries`` (mlx_foveated.py:128-169)."""
    ns = min(n_sinks, S)
    window = min(window_size, max(S - ns, 0))
    near_reserved = ns + window
    R_total = max(int(S * near_pct), near_reserved)
    far_count = S - R_total
    if far_count < 0:
        R_total = S
    mid_start = ns
    mid_end = S - window if window > 0 else S
    mid_len = max(mid_end - mid_start, 0)
    near_from_mid = min(max(R_total - near_reserved, 0), mid_len)
    R_actual = ns + near_from_mid + window
    headroom = max(int(R_actual * promo_headroom_pct), promo_headroom_min)
    near_mid_start = mid_end - near_from_mid
    return {
        "n_sinks": ns, "window": window, "near_from_mid": near_from_mid,
        "far_count": near_mid_start - mid_start, "R_actual": R_actual,
        "N_near_padded": R_actual + headroom, "mid_start": mid_start,
        "mid_end": mid_end, "near_mid_start": near_mid_start,
        "far_src_offset": mid_start,
    }


# ---------------------------------------------------------------------------
# Tier selection
# ---------------------------------------------------------------------------


def recency_indices(S: int, tb: dict):
    """Near/far positions in recency mode (mlx_foveated.py:823-843).

    near = [sinks | most recent middle | window] (ascending in each part),
    far = oldest middle, ascending.  Identical for every (b, h).
    """
    parts = [np.arange(tb["n_sinks"]),
             np.arange(tb["near_mid_start"], tb["mid_end"]),
             np.arange(S - tb["window"], S)]
    near = np.concatenate(parts).astype(np.int32)
    far = np.arange(tb["mid_start"], tb["mid_start"] + tb["far_count"], dtype=np.int32)
    return near, far


def importance_scores(k: np.ndarray, q_obs: np.ndarray) -> np.ndarray:
    """Importance of each token for one KV head (no reference implementation).

    k: (S, D) fp16, q_obs: (G, D) fp16 query heads of this KV group.
    imp[t] = sum_g softmax_t(q_g . k_t / sqrt(D)), all in fp64.
    """
    D = k.shape[-1]
    s = (q_obs.astype(np.float64) @ k.astype(np.float64).T) / math.sqrt(D)  # (G, S)
    s = s - s.max(axis=1, keepdims=True)
    e = np.exp(s)
    p = e / e.sum(axis=1, keepdims=True)
    return p.sum(axis=0)


def importance_indices(k: np.ndarray, q_obs: np.ndarray, tb: dict):
    """Near/far positions for one KV head in importance mode.

    Sinks and window are always near.  The remaining ``near_from_mid`` slots
    go to the middle tokens [mid_start, mid_end) with the largest importance;
    ties go to the lower position.  Near order: sinks, selected middle
    (ascending), window.  Far: unselected middle, ascending.
    """
    S = k.shape[0]
    imp = importance_scores(k, q_obs)
    ms, me, nfm = tb["mid_start"], tb["mid_end"], tb["near_from_mid"]
    mid = np.arange(ms, me)
    # sort by (-imp, position): lexsort uses the last key as primary
    order = np.lexsort((mid, -imp[ms:me]))
    sel = np.sort(mid[order[:nfm]])
    mask = np.zeros(S, dtype=bool)
    mask[sel] = True
    far = mid[~mask[ms:me]].astype(np.int32)
    near = np.concatenate([np.arange(tb["n_sinks"]), sel,
                           np.arange(S - tb["window"], S)]).astype(np.int32)
    return near, far


# ---------------------------------------------------------------------------
# fp8 E4M3 codec -- mlx_foveated.py:528-566 (encode), :76-91 (decode)
# ---------------------------------------------------------------------------


def fp16_to_e4m3(x: np.ndarray) -> np.ndarray:
    """Bit-level fp16 -> E4M3 exactly as ``_fp16_to_e4m3`` (mlx_foveated.py:528-566).

    Rebias -8, round-half-even 10->3 mantissa bits with carry, underflow
    (exp8<=0 after carry, or fp16 exp==0) -> signed zero, overflow (exp8>=15
    or fp16 inf/nan) -> sign|0x76.
    """
    bits = np.asarray(x, dtype=np.float16).view(np.uint16).astype(np.int32)
    sign = (bits >> 15) & 1
    exp16 = (bits >> 10) & 0x1F
    mant16 = bits & 0x3FF
    exp8_raw = exp16 - 8
    trunc = mant16 >> 7
    round_bit = (mant16 >> 6) & 1
    sticky = ((mant16 & 0x3F) != 0).astype(np.int32)
    mant3 = trunc + (round_bit & (sticky | (trunc & 1)))
    carry = (mant3 >= 8).astype(np.int32)
    mant3 = np.where(carry > 0, 0, mant3)
    exp8 = exp8_raw + carry
    under = (exp8 <= 0) | (exp16 == 0)
    over = (exp8 >= 15) | (exp16 == 31)
    exp8 = np.where(under, 0, exp8)
    mant3 = np.where(under, 0, mant3)
    exp8 = np.where(over, 14, exp8)
    mant3 = np.where(over, 6, mant3)
    return ((sign << 7) | (exp8 << 3) | mant3).astype(np.uint8)


def e4m3_to_fp16(c: np.ndarray) -> np.ndarray:
    """E4M3 -> fp16 bits as ``_e4m3_to_fp16`` (mlx_foveated.py:76-91)."""
    v = np.asarray(c).astype(np.uint32)
    sign = v >> 7
    exp8 = (v >> 3) & 0xF
    mant = v & 0x7
    exp16 = np.where(exp8 > 0, exp8 + 8, 0)
    return ((sign << 15) | (exp16 << 10) | (mant << 7)).astype(np.uint16).view(np.float16)


# ---------------------------------------------------------------------------
# INT4 V codec -- mlx_foveated.py:569-600 (encode), :94-108 (decode)
# ---------------------------------------------------------------------------


def quantize_int4(v: np.ndarray, group: Optional[int] = None):
    """Per-token (group=None) or per-group asymmetric INT4, as
    ``_quantize_int4_per_token`` (mlx_foveated.py:569-600).

    fp32 min/max; scale=(max-min)/15 (==0 -> 1); q=clip(rint((v-min)/scale),0,15);
    even dim -> low nibble.  Returns packed (..., D/2) u8, scale and zero fp16 of
    shape (...) for per-token or (..., D/group) for grouped.
    """
    v = np.asarray(v, dtype=np.float16)
    D = v.shape[-1]
    g = D if group is None else group
    fp = v.astype(np.float32).reshape(*v.shape[:-1], D // g, g)
    mn = fp.min(axis=-1, keepdims=True)
    mx_ = fp.max(axis=-1, keepdims=True)
    scale = (mx_ - mn) / np.float32(15.0)
    scale = np.where(scale == 0, np.float32(1.0), scale).astype(np.float32)
    q = np.clip(np.rint((fp - mn) / scale), 0, 15).astype(np.uint8).reshape(v.shape)
    packed = (q[..., 0::2] | (q[..., 1::2] << 4)).astype(np.uint8)
    s16 = scale[..., 0].astype(np.float16)
    z16 = mn[..., 0].astype(np.float16)
    if group is None:
        s16, z16 = s16[..., 0], z16[..., 0]
    return packed, s16, z16


def dequant_int4(packed: np.ndarray, scale: np.ndarray, zero: np.ndarray,
                 group: Optional[int] = None) -> np.ndarray:
    """INT4 -> fp16 in fp16 arithmetic (q*s then +z), as
    ``_dequant_int4_per_token`` (mlx_foveated.py:94-108)."""
    lo = (packed & 0x0F).astype(np.float16)
    hi = ((packed >> 4) & 0x0F).astype(np.float16)
    q = np.stack([lo, hi], axis=-1).reshape(*packed.shape[:-1], packed.shape[-1] * 2)
    D = q.shape[-1]
    if group is None:
        s = scale[..., None].astype(np.float16)
        z = zero[..., None].astype(np.float16)
        return (q * s + z).astype(np.float16)
    qg = q.reshape(*q.shape[:-1], D // group, group)
    out = qg * scale[..., None].astype(np.float16) + zero[..., None].astype(np.float16)
    return out.reshape(q.shape).astype(np.float16)


# ---------------------------------------------------------------------------
# TurboQuant -- turbo_constants.py:29-100, turbo_quantize.py:25-205
# ---------------------------------------------------------------------------


def turbo_rotation(d: int, seed: int = 42) -> np.ndarray:
    """turbo_constants.py:43-52: QR of RandomState(seed).randn(d,d) f32, sign-fixed."""
    rng = np.random.RandomState(seed)
    H = rng.randn(d, d).astype(np.float32)
    Q, R = np.linalg.qr(H)
    signs = np.sign(np.diag(R))
    signs[signs == 0] = 1
    return (Q * signs[np.newaxis, :]).astype(np.float32)


def turbo_qjl(d: int, seed: int = 137) -> np.ndarray:
    """turbo_constants.py:55-58: RandomState(seed).randn(d,d)/sqrt(d), stored f32."""
    rng = np.random.RandomState(seed)
    return (rng.randn(d, d).astype(np.float32) / np.sqrt(d)).astype(np.float32)


def turbo_lloyd_max(d: int, bits: int = 2, n_iters: int = 200):
    """turbo_constants.py:61-100: Lloyd-Max on N(0, 1/d), f32 results."""
    from scipy.stats import norm
    n = 2 ** bits
    sigma = 1.0 / np.sqrt(d)
    b = norm.ppf(np.linspace(0, 1, n + 1)[1:-1], scale=sigma)
    for _ in range(n_iters):
        ext = np.concatenate([[-np.inf], b, [np.inf]])
        c = np.zeros(n)
        for i in range(n):
            lo, hi = ext[i], ext[i + 1]
            p_lo = norm.pdf(lo, scale=sigma)
            p_hi = norm.pdf(hi, scale=sigma)
            prob = norm.cdf(hi, scale=sigma) - norm.cdf(lo, scale=sigma)
            if prob > 1e-15:
                c[i] = sigma ** 2 * (p_lo - p_hi) / prob
            else:
                c[i] = (lo + hi) / 2 if np.isfinite(lo + hi) else 0
        b = (c[:-1] + c[1:]) / 2
    return c.astype(np.float32), b.astype(np.float32)


def turbo_constants(d: int) -> dict:
    """``get_turbo_constants`` (turbo_constants.py:29-40)."""
    c, b = turbo_lloyd_max(d)
    return {"Pi": turbo_rotation(d), "S": turbo_qjl(d), "centroids": c, "boundaries": b}


def turbo_compress_keys(k: np.ndarray, tc: dict):
    """``turbo_compress_keys`` (turbo_quantize.py:25-91) with fp64 accumulation.

    k: (..., D) fp16.  Returns idx (...,D/4) u8 (dim 4j+i -> bits 2i),
    signs (...,D/8) u8 (bit i = dim 8j+i), norm fp16, gamma fp16.
    """
    k64 = np.asarray(k, dtype=np.float16).astype(np.float64)
    D = k64.shape[-1]
    Pi = tc["Pi"].astype(np.float64)
    S = tc["S"].astype(np.float64)
    c = tc["centroids"].astype(np.float64)
    b = tc["boundaries"].astype(np.float64)
    norm = np.sqrt(np.sum(k64 * k64, axis=-1))
    kn = k64 / np.maximum(norm, 1e-8)[..., None]
    y = kn @ Pi.T
    idx = (y >= b[0]).astype(np.uint8) + (y >= b[1]).astype(np.uint8) + (y >= b[2]).astype(np.uint8)
    r4 = idx.reshape(*idx.shape[:-1], D // 4, 4)
    idx_p = (r4[..., 0] | (r4[..., 1] << 2) | (r4[..., 2] << 4) | (r4[..., 3] << 6)).astype(np.uint8)
    k_hat = norm[..., None] * (c[idx] @ Pi)
    res = k64 - k_hat
    gamma = np.sqrt(np.sum(res * res, axis=-1))
    proj = res @ S.T
    sb = (proj >= 0).astype(np.uint8).reshape(*idx.shape[:-1], D // 8, 8)
    signs = np.zeros(sb.shape[:-1], dtype=np.uint8)
    for i in range(8):
        signs |= (sb[..., i] << i).astype(np.uint8)
    return idx_p, signs, norm.astype(np.float16), gamma.astype(np.float16)


def turbo_compress_values(v: np.ndarray, group: int = 32):
    """``turbo_compress_values`` (turbo_quantize.py:139-178), fp32 ops.

    scale = max(max|v|, 1e-8); idx = clip(rint((v/scale + 1) * 1.5), 0, 3).
    """
    v = np.asarray(v, dtype=np.float16)
    D = v.shape[-1]
    fp = v.astype(np.float32).reshape(*v.shape[:-1], D // group, group)
    sc = np.maximum(np.abs(fp).max(axis=-1), np.float32(1e-8)).astype(np.float32)
    nrm = fp / sc[..., None]
    idx = np.clip(np.rint((nrm + np.float32(1.0)) * np.float32(1.5)), 0, 3).astype(np.uint8)
    idx = idx.reshape(v.shape)
    r4 = idx.reshape(*idx.shape[:-1], D // 4, 4)
    packed = (r4[..., 0] | (r4[..., 1] << 2) | (r4[..., 2] << 4) | (r4[..., 3] << 6)).astype(np.uint8)
    return packed, sc.astype(np.float16)


def unpack_2bit(p: np.ndarray) -> np.ndarray:
    """turbo_quantize.py:278-290."""
    p = p.astype(np.uint8)
    return np.stack([p & 3, (p >> 2) & 3, (p >> 4) & 3, (p >> 6) & 3], axis=-1).reshape(
        *p.shape[:-1], p.shape[-1] * 4)


def unpack_1bit(p: np.ndarray) -> np.ndarray:
    """turbo_quantize.py:293-305 -> {-1,+1} float64."""
    bits = np.stack([(p >> i) & 1 for i in range(8)], axis=-1).reshape(*p.shape[:-1], p.shape[-1] * 8)
    return 2.0 * bits.astype(np.float64) - 1.0


TURBO_V_LEVELS = np.array([-1.0, -1.0 / 3.0, 1.0 / 3.0, 1.0], dtype=np.float32)
QJL_KERNEL = math.sqrt(math.pi / 2.0)   # foveated_attn.metal:518 (1.2533141/D)
QJL_DEQUANT = 1.0                       # turbo_quantize.py:129 (signs@S / D)


def turbo_dequant_values(packed: np.ndarray, scales: np.ndarray, group: int = 32) -> np.ndarray:
    """turbo_quantize.py:181-205: level[idx] * scale, fp32 -> fp16."""
    idx = unpack_2bit(packed)
    lv = TURBO_V_LEVELS[idx]
    D = idx.shape[-1]
    g = lv.reshape(*lv.shape[:-1], D // group, group) * scales.astype(np.float32)[..., None]
    return g.reshape(lv.shape).astype(np.float16)


def turbo_far_scores(q: np.ndarray, idx: np.ndarray, signs: np.ndarray, norm: np.ndarray,
                     gamma: np.ndarray, tc: dict, qjl_coef: float = QJL_KERNEL) -> np.ndarray:
    """Far scores directly on codes (foveated_attn.metal:486-521,684-688), fp64.

    q: (G, D) fp16, codes (F, ...).  score = (|k| * q_rot.c[idx]
    + coef/D * gamma * q_sketch.sign) / sqrt(D), with q_rot = q Pi^T and
    q_sketch = q S^T computed from the unscaled query.  Returns (G, F).
    """
    q64 = q.astype(np.float64)
    D = q64.shape[-1]
    q_rot = q64 @ tc["Pi"].astype(np.float64).T
    q_sk = q64 @ tc["S"].astype(np.float64).T
    cv = tc["centroids"].astype(np.float64)[unpack_2bit(idx)]       # (F, D)
    sg = unpack_1bit(signs)                                           # (F, D)
    mse = norm.astype(np.float64)[None, :] * (q_rot @ cv.T)
    qjl = (qjl_coef / D) * gamma.astype(np.float64)[None, :] * (q_sk @ sg.T)
    return (mse + qjl) / math.sqrt(D)


# ---------------------------------------------------------------------------
# Layer compression -- _assign_and_build_layer (mlx_foveated.py:799-944)
# ---------------------------------------------------------------------------


def compress_layer(K: np.ndarray, V: np.ndarray, cfg: dict, q_obs: Optional[np.ndarray] = None,
                   tc: Optional[dict] = None) -> dict:
    """Restates ``_assign_and_build_layer`` (mlx_foveated.py:799-944).

    K, V: (B, Hk, S, D) fp16.  cfg keys: near_pct, n_sinks, window_size,
    promo_headroom_pct, promo_headroom_min, compress_method ('fp8'|'turbo'),
    select ('recency'|'importance'), v_group (None|32).  ``q_obs``
    (B, Hq, D) fp16 is required for importance mode.

    near_valid is (B, Hk) (the reference keeps (Hk,), identical at B=1).
    """
    K = np.asarray(K, dtype=np.float16)
    V = np.asarray(V, dtype=np.float16)
    B, Hk, S, D = K.shape
    tb = tier_boundaries(S, cfg.get("near_pct", 0.10), cfg.get("n_sinks", 4),
                         cfg.get("window_size", 32), cfg.get("promo_headroom_pct", 0.5),
                         cfg.get("promo_headroom_min", 8))
    R, Np, F = tb["R_actual"], tb["N_near_padded"], tb["far_count"]
    near_idx = np.full((B, Hk, Np), -1, dtype=np.int32)
    far_idx = np.zeros((B, Hk, F), dtype=np.int32)
    if cfg.get("select", "recency") == "importance":
        Hq = q_obs.shape[1]
        G = Hq // Hk
        for b in range(B):
            for h in range(Hk):
                n, f = importance_indices(K[b, h], q_obs[b, h * G:(h + 1) * G], tb)
                near_idx[b, h, :R] = n
                far_idx[b, h] = f
    else:
        n, f = recency_indices(S, tb)
        near_idx[:, :, :R] = n
        far_idx[:, :, :] = f
    gi = near_idx[:, :, :R]
    near_k = np.zeros((B, Hk, Np, D), dtype=np.float16)
    near_v = np.zeros((B, Hk, Np, D), dtype=np.float16)
    near_k[:, :, :R] = np.take_along_axis(K, gi[..., None].astype(np.int64), axis=2)
    near_v[:, :, :R] = np.take_along_axis(V, gi[..., None].astype(np.int64), axis=2)
    arc_k = np.take_along_axis(K, far_idx[..., None].astype(np.int64), axis=2)
    arc_v = np.take_along_axis(V, far_idx[..., None].astype(np.int64), axis=2)
    out = {"tb": tb, "near_k": near_k, "near_v": near_v, "near_idx": near_idx,
           "near_valid": np.full((B, Hk), R, dtype=np.int32), "far_idx": far_idx,
           "archive_k": arc_k, "archive_v": arc_v,
           "compress_method": cfg.get("compress_method", "fp8"),
           "v_group": cfg.get("v_group", None)}
    if out["compress_method"] == "turbo":
        tc = tc if tc is not None else turbo_constants(D)
        ki, ks, kn, kg = turbo_compress_keys(arc_k, tc)
        vp, vs = turbo_compress_values(arc_v)
        out.update(turbo_k_idx=ki, turbo_k_signs=ks, turbo_k_norm=kn, turbo_k_gamma=kg,
                   turbo_v_packed=vp, turbo_v_scale=vs, tc=tc)
    else:
        out["far_k"] = fp16_to_e4m3(arc_k)
        out["far_v"], out["far_v_scale"], out["far_v_zero"] = quantize_int4(arc_v, out["v_group"])
    return out


# ---------------------------------------------------------------------------
# Decode attention oracle (attend + spike semantics)
# ---------------------------------------------------------------------------


def prescaled_query(q: np.ndarray) -> np.ndarray:
    """q(f16) * f32(1/sqrt(D)) in fp32, as the kernel pre-scales (foveated_attn.metal:258-261)."""
    D = q.shape[-1]
    return q.astype(np.float32) * np.float32(1.0 / math.sqrt(D))


def decode_attend(layer: dict, q: np.ndarray, dec_k: Optional[np.ndarray] = None,
                  dec_v: Optional[np.ndarray] = None, spike_margin: float = 0.5,
                  qjl_coef: float = QJL_KERNEL):
    """Fused decode attention + spike flags, per-(b, h) ``near_valid``.

    Output follows ``attend`` (mlx_foveated.py:239-312): far tier dequantised
    to fp16 (fp8 K exact, INT4 V in fp16 arithmetic), concatenated with the
    valid near rows and the decode buffer, softmax attention in fp64 with scale
    1/sqrt(D).  Turbo far scores are taken on codes (see ``turbo_far_scores``).

    Spikes follow foveated_attn.metal:269-431: min_near over near + decode
    scores, max_far/argmax (earliest index on ties) over far scores,
    flag = max_far > min_near + margin, token = far-local argmax or -1.

    q: (B, Hq, D) fp16; dec_k/dec_v: (B, Hk, n, D) fp16 or None.
    Returns out (B,Hq,D) f64, flags (B,Hq) i32, tokens (B,Hq) i32, and a dict
    with max_far / min_near / second_far for tie diagnostics.
    """
    q = np.asarray(q, dtype=np.float16)
    B, Hq, D = q.shape
    Hk = layer["near_k"].shape[1]
    G = Hq // Hk
    method = layer.get("compress_method", "fp8")
    if method == "turbo":
        far_v_all = turbo_dequant_values(layer["turbo_v_packed"], layer["turbo_v_scale"])
    else:
        far_k_all = e4m3_to_fp16(layer["far_k"])
        far_v_all = dequant_int4(layer["far_v"], layer["far_v_scale"], layer["far_v_zero"],
                                 layer.get("v_group"))
    qs = prescaled_query(q).astype(np.float64)
    out = np.zeros((B, Hq, D), dtype=np.float64)
    flags = np.zeros((B, Hq), dtype=np.int32)
    tokens = np.full((B, Hq), -1, dtype=np.int32)
    diag = {k: np.zeros((B, Hq)) for k in ("max_far", "min_near", "second_far")}
    for b in range(B):
        for h in range(Hk):
            nv = int(layer["near_valid"][b, h])
            nk = layer["near_k"][b, h, :nv].astype(np.float64)
            nvv = layer["near_v"][b, h, :nv].astype(np.float64)
            if dec_k is not None and dec_k.shape[2] > 0:
                nk = np.concatenate([nk, dec_k[b, h].astype(np.float64)])
                nvv = np.concatenate([nvv, dec_v[b, h].astype(np.float64)])
            qg = qs[b, h * G:(h + 1) * G]                      # (G, D)
            s_near = qg @ nk.T                                  # (G, Nn)
            if method == "turbo":
                s_far = turbo_far_scores(q[b, h * G:(h + 1) * G], layer["turbo_k_idx"][b, h],
                                         layer["turbo_k_signs"][b, h], layer["turbo_k_norm"][b, h],
                                         layer["turbo_k_gamma"][b, h], layer["tc"], qjl_coef)
            else:
                s_far = qg @ far_k_all[b, h].astype(np.float64).T
            fv = far_v_all[b, h].astype(np.float64)
            s = np.concatenate([s_near, s_far], axis=1)
            vv = np.concatenate([nvv, fv])
            if s.shape[1] > 0:
                m = s.max(axis=1, keepdims=True)
                p = np.exp(s - m)
                out[b, h * G:(h + 1) * G] = (p @ vv) / p.sum(axis=1, keepdims=True)
            for g in range(G):
                hq = h * G + g
                mn = s_near[g].min() if s_near.shape[1] else np.inf
                if s_far.shape[1]:
                    am = int(np.argmax(s_far[g]))        # first max = earliest index
                    mf = s_far[g, am]
                    srt = np.sort(s_far[g])
                    diag["second_far"][b, hq] = srt[-2] if srt.size > 1 else -np.inf
                    tokens[b, hq] = am
                else:
                    mf = -np.inf
                diag["max_far"][b, hq] = mf
                diag["min_near"][b, hq] = mn
                flags[b, hq] = 1 if mf > mn + spike_margin else 0
    return out, flags, tokens, diag


# ---------------------------------------------------------------------------
# The reference's CPU attend in its own precision (timed CPU baseline)
# ---------------------------------------------------------------------------

_E4M3_LUT = None


def _e4m3_lut() -> np.ndarray:
    global _E4M3_LUT
    if _E4M3_LUT is None:
        _E4M3_LUT = e4m3_to_fp16(np.arange(256, dtype=np.uint8))
    return _E4M3_LUT


def reference_attend_f32(layer: dict, q: np.ndarray, dec_k: Optional[np.ndarray] = None,
                         dec_v: Optional[np.ndarray] = None, threads: int = 1) -> np.ndarray:
    """``MLXFoveatedLayer.attend`` (mlx_foveated.py:239-278) in the reference's
    own precision, as the CPU baseline the fused kernel is timed against:
    far K E4M3 -> fp16 (a 256-entry table lookup, the same bits as
    ``_e4m3_to_fp16``), far V INT4 -> fp16 in fp16 arithmetic
    (``_dequant_int4_per_token``: code*scale and +zero, each rounded to fp16),
    [valid near | decode | far] concatenated, K/V shared by the G query heads
    of a group (the values ``mx.repeat`` replicates, converted once), then fp32
    softmax attention with scale 1/sqrt(D) (MLX's CPU SDPA computes fp16
    inputs in fp32).  No spike tracking or diagnostics: this is the work the
    reference's CPU path does per decode step.  fp8 far tier, per-token V
    scales.  The (b, kv head) streams are independent; ``threads`` > 1 runs
    them on a thread pool (NumPy releases the GIL in these kernels; keep BLAS
    single-threaded then).  Returns (B, Hq, D) f32.
    """
    q = np.asarray(q, dtype=np.float16)
    B, Hq, D = q.shape
    Hk = layer["near_k"].shape[1]
    G = Hq // Hk
    lut = _e4m3_lut()
    nv = int(np.max(layer["near_valid"]))
    scale = np.float32(1.0 / math.sqrt(D))
    out = np.empty((B, Hq, D), dtype=np.float32)
    f32, f16 = np.float32, np.float16

    def stream(bh):
        b, h = divmod(bh, Hk)
        fk = lut[layer["far_k"][b, h]]
        pk = layer["far_v"][b, h]
        codes = np.empty(pk.shape[:-1] + (2 * pk.shape[-1],), dtype=f32)
        codes[:, 0::2] = pk & 0x0F
        codes[:, 1::2] = pk >> 4
        sc = layer["far_v_scale"][b, h][:, None].astype(f32)
        ze = layer["far_v_zero"][b, h][:, None].astype(f32)
        # fp16 arithmetic: each operation's exact fp32 result rounded to fp16
        fv = ((codes * sc).astype(f16).astype(f32) + ze).astype(f16)
        ks = [layer["near_k"][b, h, :nv]]
        vs = [layer["near_v"][b, h, :nv]]
        if dec_k is not None and dec_k.shape[2] > 0:
            ks.append(dec_k[b, h])
            vs.append(dec_v[b, h])
        k32 = np.concatenate(ks + [fk]).astype(f32)
        v32 = np.concatenate(vs + [fv]).astype(f32)
        qg = q[b, h * G:(h + 1) * G].astype(f32) * scale
        sc_ = qg @ k32.T
        p = np.exp(sc_ - sc_.max(axis=1, keepdims=True))
        out[b, h * G:(h + 1) * G] = (p @ v32) / p.sum(axis=1, keepdims=True)

    if threads > 1:
        from concurrent.futures import ThreadPoolExecutor
        with ThreadPoolExecutor(threads) as ex:
            list(ex.map(stream, range(B * Hk)))
    else:
        for bh in range(B * Hk):
            stream(bh)
    return out


# ---------------------------------------------------------------------------
# Split-sequence combine (multi-GPU; no reference counterpart)
# ---------------------------------------------------------------------------


def combine_partials(m, l, o, min_near, max_far, arg_far, spike_margin):
    """Merge per-shard softmax partials in shard order.

    m, l, min_near, max_far: (P, N) ; o: (P, N, D) ; arg_far: (P, N) int
    (global far index, -1 if none).  Rescale by exp(m_p - max m); spike
    argmax from the first shard holding the strict maximum
    (foveated_attn.metal:399-431 semantics applied across shards).
    """
    P = m.shape[0]
    M = np.max(m, axis=0)
    w = np.where(np.isfinite(m), np.exp(m - M[None]), 0.0)
    L = np.sum(w * l, axis=0)
    O = np.sum(w[..., None] * o, axis=0)
    out = np.where(L[..., None] > 0, O / np.where(L > 0, L, 1)[..., None], 0.0)
    mn = np.min(min_near, axis=0)
    mf = np.full(m.shape[1], -np.inf)
    tok = np.full(m.shape[1], -1, dtype=np.int64)
    for p in range(P):
        better = max_far[p] > mf
        mf = np.where(better, max_far[p], mf)
        tok = np.where(better, arg_far[p], tok)
    flags = (mf > mn + spike_margin).astype(np.int32)
    return out, flags, tok.astype(np.int32)


# ---------------------------------------------------------------------------
# Promotion drain filter -- promotion_pipeline.cpp:99-175
# ---------------------------------------------------------------------------


class DrainFilter:
    """Host restatement of ``PromotionPipeline::drain_spikes``.

    Filters in order: flag==0, GQA dedup (first q head per (b, kv head) per
    call), per-(layer, b, kv head) cooldown, far-local -> position, position
    dedup, archive lookup; at most ``max_per_drain`` records per call.  The
    reference keys GQA dedup and cooldown by kv head only and promotes batch 0
    only (promotion_pipeline.cpp:117-139,230); with B=1 the two agree.
    """

    def __init__(self, cooldown_steps: int = 5, max_per_drain: int = 8):
        self.cooldown = cooldown_steps
        self.budget = max_per_drain
        self.last = {}
        self.promoted = set()
        self.stats = {"spikes_detected": 0, "spikes_queued": 0, "spikes_deduplicated": 0,
                      "spikes_cooled_down": 0}

    def drain(self, layer, flags, tokens, far_idx, step, arc_len=None):
        B, Hq = flags.shape
        Hk, F = far_idx.shape[1], far_idx.shape[2]
        G = Hq // Hk if Hk else 1
        seen = set()
        out = []
        for b in range(B):
            for hq in range(Hq):
                if len(out) >= self.budget:
                    return out
                if flags[b, hq] == 0:
                    continue
                h = hq // G
                if (b, h) in seen:
                    continue
                seen.add((b, h))
                self.stats["spikes_detected"] += 1
                key = (layer, b, h)
                if key in self.last and step - self.last[key] < self.cooldown:
                    self.stats["spikes_cooled_down"] += 1
                    continue
                self.last[key] = step
                fl = int(tokens[b, hq])
                if fl < 0 or fl >= F:
                    continue
                pos = int(far_idx[b, h, fl])
                dk = (layer, b, h, pos)
                if dk in self.promoted:
                    self.stats["spikes_deduplicated"] += 1
                    continue
                self.promoted.add(dk)
                if arc_len is not None and fl >= arc_len:
                    continue
                out.append((layer, b, h, fl, pos))
                self.stats["spikes_queued"] += 1
        return out


def shard_tier_positions(S: int, lo: int, hi: int, tb: dict):
    """Near / far positions of the global recency tiers that fall in the
    shard [lo, hi) (sequence split; no reference counterpart).  Returns
    (near_positions, far_positions, far_index_offset) with the far offset the
    global far-local index of the shard's first far token."""
    near, far = recency_indices(S, tb)
    n = near[(near >= lo) & (near < hi)]
    f = far[(far >= lo) & (far < hi)]
    off = int(f[0] - tb["mid_start"]) if f.size else 0
    return n.astype(np.int32), f.astype(np.int32), off


def decode_partials(layer: dict, q: np.ndarray, dec_k=None, dec_v=None, far_offset: int = 0):
    """Per (b, q head) partial softmax record of this tier shard:
    m, l (sum exp(s - m)), o (sum exp(s - m) v, unnormalised), min_near,
    max_far and its global far index (earliest on ties) or -1."""
    q = np.asarray(q, dtype=np.float16)
    B, Hq, D = q.shape
    Hk = layer["near_k"].shape[1]
    G = Hq // Hk
    fk = e4m3_to_fp16(layer["far_k"])
    fv = dequant_int4(layer["far_v"], layer["far_v_scale"], layer["far_v_zero"], layer.get("v_group"))
    qs = prescaled_query(q).astype(np.float64)
    N = B * Hq
    m = np.full(N, -np.inf); l = np.zeros(N); o = np.zeros((N, D))
    mn = np.full(N, np.inf); mf = np.full(N, -np.inf); arg = np.full(N, -1, dtype=np.int64)
    for b in range(B):
        for h in range(Hk):
            nv = int(layer["near_valid"][b, h])
            nk = layer["near_k"][b, h, :nv].astype(np.float64)
            nvv = layer["near_v"][b, h, :nv].astype(np.float64)
            if dec_k is not None and dec_k.shape[2] > 0:
                nk = np.concatenate([nk, dec_k[b, h].astype(np.float64)])
                nvv = np.concatenate([nvv, dec_v[b, h].astype(np.float64)])
            qg = qs[b, h * G:(h + 1) * G]
            sn = qg @ nk.T
            sf = qg @ fk[b, h].astype(np.float64).T
            sc = np.concatenate([sn, sf], axis=1)
            vv = np.concatenate([nvv, fv[b, h].astype(np.float64)])
            for g in range(G):
                i = b * Hq + h * G + g
                if sc.shape[1]:
                    m[i] = sc[g].max()
                    p = np.exp(sc[g] - m[i])
                    l[i] = p.sum()
                    o[i] = p @ vv
                if sn.shape[1]:
                    mn[i] = sn[g].min()
                if sf.shape[1]:
                    a = int(np.argmax(sf[g]))
                    mf[i] = sf[g, a]
                    arg[i] = a + far_offset
    return m, l, o, mn, mf, arg
