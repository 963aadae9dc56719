"""Generate the golden fixtures in this directory from the reference's own
Python CPU path.

Usage:  python tests/golden/make_golden.py --reference <path to samfurr/foveated_kv checkout>

The reference needs MLX, which cannot be installed here; ``mlx_shim/``
provides the handful of ``mlx.core`` operations that ``mlx_foveated.py``,
``turbo_quantize.py`` and ``turbo_constants.py`` use, on NumPy.  The
reference modules are imported unmodified from the checkout (its package
``__init__`` is bypassed because it pulls in unrelated modules).  Outputs:

  fp8_table.npz          every fp16 bit pattern -> reference E4M3 code, and
                         every code -> reference fp16 (exhaustive)
  int4_cases.npz         reference per-token INT4 on random + edge rows
  tier_boundaries.json   reference tier_boundaries for a grid of S/configs
  turbo_constants.npz    reference Pi, S, centroids, boundaries for d=64,128
  turbo_codes.npz        reference turbo_compress_keys/values (fp32 path)
  layer_c0_fp8.npz       reference _assign_and_build_layer, c0 shape, recency
  layer_small_turbo.npz  reference _assign_and_build_layer, turbo, small
  layer_hashes.json      sha256 of every output of _assign_and_build_layer for
                         the larger configs (inputs are regenerated from seed)
  attend_c0.npz          reference attend() (dequant -> SDPA via the shim's
                         float32 SDPA) for c0 + the tier it attended over

Nothing at run time (tests, smoke, bench) reads the reference; only these
fixtures.
"""

from __future__ import annotations

import argparse
import hashlib
import importlib
import json
import os
import sys
import types

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from foveated_kv_b200.synthetic import numpy_workload, CONFIGS  # noqa: E402


def load_reference(ref_root: str):
    sys.path.insert(0, os.path.join(HERE, "mlx_shim"))
    src = os.path.join(ref_root, "src", "foveated_kv")
    pkg = types.ModuleType("foveated_kv")
    pkg.__path__ = [src]
    sys.modules["foveated_kv"] = pkg
    mf = importlib.import_module("foveated_kv.mlx_foveated")
    tq = importlib.import_module("foveated_kv.turbo_quantize")
    tcm = importlib.import_module("foveated_kv.turbo_constants")
    return mf, tq, tcm


def sha(a) -> str:
    a = np.ascontiguousarray(np.asarray(a))
    return hashlib.sha256(a.tobytes() + str(a.dtype).encode() + str(a.shape).encode()).hexdigest()


LAYER_FIELDS = ["near_k", "near_v", "near_idx", "near_valid", "far_k", "far_v",
                "far_v_scale", "far_v_zero", "far_idx", "archive_k", "archive_v"]
TURBO_FIELDS = ["turbo_far_k_indices", "turbo_far_k_signs", "turbo_far_k_norm",
                "turbo_far_k_gamma", "turbo_far_v_packed", "turbo_far_v_scale"]


def build_layer(mf, k, v, **cfgkw):
    cfg = mf.MLXTierConfig(**cfgkw)
    cache = mf.MLXFoveatedKVCache(cfg)
    B, H, S, D = k.shape
    return cache._assign_and_build_layer(k, v, B, H, S, D)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    args = ap.parse_args()
    mf, tq, tcm = load_reference(args.reference)

    # --- fp8 codec, exhaustive -------------------------------------------
    allbits = np.arange(65536, dtype=np.uint32).astype(np.uint16).view(np.float16)
    enc = np.asarray(mf._fp16_to_e4m3(allbits)).astype(np.uint8)
    dec = np.asarray(mf._e4m3_to_fp16(np.arange(256, dtype=np.uint8))).view(np.uint16)
    np.savez_compressed(os.path.join(HERE, "fp8_table.npz"), encode=enc, decode_bits=dec)

    # --- INT4 per token ---------------------------------------------------
    rs = np.random.RandomState(7)
    x = rs.standard_normal((1, 2, 64, 64)).astype(np.float16)
    x[0, 0, 0] = 0                                 # all-zero row -> scale 1
    x[0, 0, 1] = np.float16(3.5)                   # constant row
    x[0, 0, 2] = (rs.standard_normal(64) * 300).astype(np.float16)   # wide range
    x[0, 0, 3, ::2] = np.float16(-1.0)             # exact ties
    x[0, 0, 3, 1::2] = np.float16(1.0)
    x[0, 1, 5] = (np.arange(64) / 4.0 - 8).astype(np.float16)        # half-integer codes
    p, s, z = mf._quantize_int4_per_token(x)
    np.savez_compressed(os.path.join(HERE, "int4_cases.npz"), x=x, packed=np.asarray(p),
                        scale=np.asarray(s), zero=np.asarray(z))

    # --- tier boundaries --------------------------------------------------
    tbs = []
    for S in [0, 1, 3, 4, 5, 8, 36, 37, 100, 255, 256, 1000, 1024, 4096, 16384, 32768, 1 << 20]:
        for cfg in [dict(), dict(window_size=64), dict(window_size=128),
                    dict(near_pct=0.05), dict(near_pct=0.3, n_sinks=0, window_size=0),
                    dict(promo_headroom_pct=0.25, promo_headroom_min=4)]:
            c = mf.MLXTierConfig(**cfg)
            tbs.append({"S": S, "cfg": cfg, "tb": c.tier_boundaries(S)})
    with open(os.path.join(HERE, "tier_boundaries.json"), "w") as f:
        json.dump(tbs, f, indent=0)

    # --- turbo constants + codes -----------------------------------------
    consts = {}
    for d in (64, 128):
        c, b = tcm._lloyd_max_centroids(d, bits=2)
        consts[f"Pi_{d}"] = tcm._rotation_matrix(d, 42)
        consts[f"S_{d}"] = tcm._qjl_matrix(d, 137).astype(np.float32)
        consts[f"centroids_{d}"] = c
        consts[f"boundaries_{d}"] = b
    np.savez_compressed(os.path.join(HERE, "turbo_constants.npz"), **consts)

    tc = tcm.get_turbo_constants(128)
    kk = rs.standard_normal((1, 2, 96, 128)).astype(np.float16)
    vv = rs.standard_normal((1, 2, 96, 128)).astype(np.float16)
    ki, ks, kn, kg = tq.turbo_compress_keys(kk, tc)
    vp, vs = tq.turbo_compress_values(vv)
    np.savez_compressed(os.path.join(HERE, "turbo_codes.npz"), k=kk, v=vv, k_idx=ki, k_signs=ks,
                        k_norm=kn, k_gamma=kg, v_packed=vp, v_scale=vs)

    # --- layers -----------------------------------------------------------
    c0 = CONFIGS["c0"]
    w = numpy_workload(100, c0["B"], c0["Hk"], c0["Hq"], c0["S"], c0["D"], c0["n_dec"])
    lay = build_layer(mf, w["k"], w["v"], near_pct=0.10, n_sinks=4, window_size=64)
    np.savez_compressed(os.path.join(HERE, "layer_c0_fp8.npz"),
                        **{f: np.asarray(getattr(lay, f)) for f in LAYER_FIELDS})
    q4 = w["q"][:, :, None, :]
    out = lay.attend(q4)
    np.savez_compressed(os.path.join(HERE, "attend_c0.npz"), q=w["q"], out=np.asarray(out)[:, :, 0])

    wt = numpy_workload(101, 1, 2, 14, 512, 64, 0)
    lt = build_layer(mf, wt["k"], wt["v"], near_pct=0.10, n_sinks=4, window_size=32,
                     compress_method="turbo")
    np.savez_compressed(os.path.join(HERE, "layer_small_turbo.npz"),
                        **{f: np.asarray(getattr(lt, f)) for f in LAYER_FIELDS + TURBO_FIELDS})

    hashes = {}
    for name, seed in [("c1_1k", 200)]:
        c = CONFIGS[name]
        wl = numpy_workload(seed, c["B"], c["Hk"], c["Hq"], c["S"], c["D"], 0)
        lay = build_layer(mf, wl["k"], wl["v"], near_pct=c["near_pct"], n_sinks=c["n_sinks"],
                          window_size=c["window_size"])
        hashes[name] = {"seed": seed, **{f: sha(getattr(lay, f)) for f in LAYER_FIELDS}}
    with open(os.path.join(HERE, "layer_hashes.json"), "w") as f:
        json.dump(hashes, f, indent=1)
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main()
