"""Pin the CPU oracle against fixtures produced by the reference's own Python
CPU path (tests/golden/make_golden.py) and re-pin the reference's
known-answer / property tests (tests/test_mlx_foveated.py,
tests/test_turbo_quantize.py of the reference)."""

import hashlib
import json
import os

import numpy as np
import pytest

from oracle import fkv_oracle as O
from foveated_kv_b200.synthetic import numpy_workload, CONFIGS

GOLD = os.path.join(os.path.dirname(__file__), "golden")


def _bits(a):
    a = np.ascontiguousarray(a)
    return a.view(np.uint16) if a.dtype == np.float16 else a


def test_fp8_encode_exhaustive(golden):
    t = golden("fp8_table.npz")
    allb = np.arange(65536, dtype=np.uint32).astype(np.uint16).view(np.float16)
    assert np.array_equal(O.fp16_to_e4m3(allb), t["encode"])


def test_fp8_decode_exhaustive(golden):
    t = golden("fp8_table.npz")
    dec = O.e4m3_to_fp16(np.arange(256, dtype=np.uint8)).view(np.uint16)
    assert np.array_equal(dec, t["decode_bits"])


def test_fp8_never_emits_subnormal_or_nan():
    allb = np.arange(65536, dtype=np.uint32).astype(np.uint16).view(np.float16)
    c = O.fp16_to_e4m3(allb)
    exp8, mant = (c >> 3) & 0xF, c & 7
    assert not np.any((exp8 == 0) & (mant != 0))
    assert not np.any(exp8 == 15)          # saturation is 0x76 (224); 0x77 (240) is a rounded normal
    assert (c & 0x7F).max() == 0x77


def test_int4_cases(golden):
    c = golden("int4_cases.npz")
    p, s, z = O.quantize_int4(c["x"])
    assert np.array_equal(p, c["packed"])
    assert np.array_equal(_bits(s), _bits(c["scale"]))
    assert np.array_equal(_bits(z), _bits(c["zero"]))


def test_tier_boundaries_grid():
    with open(os.path.join(GOLD, "tier_boundaries.json")) as f:
        tbs = json.load(f)
    for e in tbs:
        assert O.tier_boundaries(e["S"], **e["cfg"]) == e["tb"], e


def test_tier_sizes_known_answer():
    # reference tests/test_mlx_foveated.py:235-249: S=1000 -> 100 near, 900 far
    tb = O.tier_boundaries(1000, 0.10, 4, 32)
    assert tb["R_actual"] == 100 and tb["far_count"] == 900
    assert tb["N_near_padded"] > 100


@pytest.mark.parametrize("d", [64, 128])
def test_turbo_constants(golden, d):
    t = golden("turbo_constants.npz")
    mine = O.turbo_constants(d)
    for k in ("Pi", "S", "centroids", "boundaries"):
        assert np.array_equal(mine[k], t[f"{k}_{d}"]), k
    Pi = mine["Pi"].astype(np.float64)
    assert np.allclose(Pi @ Pi.T, np.eye(d), atol=1e-5)
    c = mine["centroids"]
    assert np.allclose(c, -c[::-1], atol=1e-6) and np.all(np.diff(c) > 0)
    assert np.all(np.diff(mine["boundaries"]) > 0)


def test_turbo_codes_vs_reference_fp32_path(golden):
    t = golden("turbo_codes.npz")
    tc = {k: golden("turbo_constants.npz")[f"{k}_128"] for k in ("Pi", "S", "centroids", "boundaries")}
    ki, ks, kn, kg = O.turbo_compress_keys(t["k"], tc)
    assert np.array_equal(ki, t["k_idx"])
    assert np.array_equal(ks, t["k_signs"])
    assert np.array_equal(_bits(kn), _bits(t["k_norm"]))
    assert np.array_equal(_bits(kg), _bits(t["k_gamma"]))
    vp, vs = O.turbo_compress_values(t["v"])
    assert np.array_equal(vp, t["v_packed"])
    assert np.array_equal(_bits(vs), _bits(t["v_scale"]))


def test_turbo_packing_known_answers():
    # reference tests/test_turbo_quantize.py:85-109
    orig = np.array([0, 1, 2, 3, 3, 2, 1, 0], dtype=np.uint8)
    packed = (orig[0::4] | (orig[1::4] << 2) | (orig[2::4] << 4) | (orig[3::4] << 6)).astype(np.uint8)
    assert np.array_equal(O.unpack_2bit(packed[None])[0], orig)
    bits = np.array([1, 0, 1, 1, 0, 0, 1, 0], dtype=np.uint8)
    byte = np.uint8(sum(int(b) << i for i, b in enumerate(bits)))
    assert np.array_equal(O.unpack_1bit(np.array([[byte]]))[0], 2.0 * bits - 1.0)


def test_layer_c0_fp8_bit_exact(golden):
    L = golden("layer_c0_fp8.npz")
    c = CONFIGS["c0"]
    w = numpy_workload(100, c["B"], c["Hk"], c["Hq"], c["S"], c["D"], c["n_dec"])
    mine = O.compress_layer(w["k"], w["v"], dict(window_size=64))
    for f in L.files:
        ref = L[f]
        if f == "near_valid":      # reference keeps (Hk,), shared across batch
            assert np.all(mine[f] == ref[None, :])
            continue
        assert np.array_equal(_bits(mine[f]), _bits(ref)), f


def test_layer_turbo_bit_exact(golden):
    L = golden("layer_small_turbo.npz")
    w = numpy_workload(101, 1, 2, 14, 512, 64, 0)
    mine = O.compress_layer(w["k"], w["v"], dict(window_size=32, compress_method="turbo"))
    pairs = {"turbo_far_k_indices": "turbo_k_idx", "turbo_far_k_signs": "turbo_k_signs",
             "turbo_far_k_norm": "turbo_k_norm", "turbo_far_k_gamma": "turbo_k_gamma",
             "turbo_far_v_packed": "turbo_v_packed", "turbo_far_v_scale": "turbo_v_scale"}
    for f in ["near_k", "near_v", "near_idx", "far_idx", "archive_k", "archive_v"]:
        assert np.array_equal(_bits(mine[f]), _bits(L[f])), f
    for rf, mf in pairs.items():
        assert np.array_equal(_bits(mine[mf]), _bits(L[rf])), rf


def _sha(a):
    a = np.ascontiguousarray(np.asarray(a))
    return hashlib.sha256(a.tobytes() + str(a.dtype).encode() + str(a.shape).encode()).hexdigest()


def test_layer_c1_1k_hashes():
    with open(os.path.join(GOLD, "layer_hashes.json")) as f:
        H = json.load(f)["c1_1k"]
    c = CONFIGS["c1_1k"]
    w = numpy_workload(H["seed"], c["B"], c["Hk"], c["Hq"], c["S"], c["D"], 0)
    mine = O.compress_layer(w["k"], w["v"], dict(near_pct=c["near_pct"], n_sinks=c["n_sinks"],
                                                   window_size=c["window_size"]))
    for f, h in H.items():
        if f == "seed":
            continue
        val = mine[f][0] if f == "near_valid" else mine[f]
        assert _sha(val) == h, f


def test_attend_c0_vs_reference_attend(golden):
    A = golden("attend_c0.npz")
    c = CONFIGS["c0"]
    w = numpy_workload(100, c["B"], c["Hk"], c["Hq"], c["S"], c["D"], c["n_dec"])
    lay = O.compress_layer(w["k"], w["v"], dict(window_size=64))
    out, _, _, _ = O.decode_attend(lay, w["q"])
    ref = A["out"].astype(np.float64)
    assert np.abs(out - ref).max() < 2e-3
    cos = (out * ref).sum() / np.sqrt((out * out).sum() * (ref * ref).sum())
    assert cos > 0.9999


def test_zero_rows_preserved():
    # reference tests/test_mlx_foveated.py:146-151,201-206
    z = np.zeros((1, 1, 4, 64), dtype=np.float16)
    assert np.all(O.e4m3_to_fp16(O.fp16_to_e4m3(z)) == 0)
    p, s, zz = O.quantize_int4(z)
    assert np.all(O.dequant_int4(p, s, zz) == 0)


def test_importance_selection_properties():
    w = numpy_workload(5, 1, 2, 8, 300, 64, 0)
    tb = O.tier_boundaries(300, 0.2, 4, 16)
    for h in range(2):
        near, far = O.importance_indices(w["k"][0, h], w["q_obs"][0, 4 * h:4 * h + 4], tb)
        assert len(near) == tb["R_actual"] and len(far) == tb["far_count"]
        assert np.array_equal(np.sort(np.concatenate([near, far])), np.arange(300))
        assert np.array_equal(near[:4], np.arange(4))
        assert np.array_equal(near[-16:], np.arange(284, 300))
        imp = O.importance_scores(w["k"][0, h], w["q_obs"][0, 4 * h:4 * h + 4])
        sel = near[4:-16]
        assert imp[sel].min() >= imp[far].max()
        assert np.all(np.diff(far) > 0) and np.all(np.diff(sel) > 0)


def test_combine_partials_matches_single_pass():
    rs = np.random.RandomState(0)
    s = rs.standard_normal((3, 50))
    v = rs.standard_normal((50, 8))
    parts = np.array_split(np.arange(50), 4)
    m = np.array([[s[h, p].max() for h in range(3)] for p in parts])
    l = np.array([[np.exp(s[h, p] - s[h, p].max()).sum() for h in range(3)] for p in parts])
    o = np.array([[(np.exp(s[h, p] - s[h, p].max()) @ v[p]) for h in range(3)] for p in parts])
    inf = np.full((4, 3), np.inf)
    out, fl, tok = O.combine_partials(m, l, o, inf, -inf, np.full((4, 3), -1), 0.5)
    p = np.exp(s - s.max(1, keepdims=True))
    assert np.allclose(out, (p @ v) / p.sum(1, keepdims=True))


@pytest.mark.parametrize("d", [64, 128])
def test_product_turbo_constants_match_reference(golden, d):
    """The package's own host-side constants equal the reference's."""
    from foveated_kv_b200.turbo_constants import host_constants
    t = golden("turbo_constants.npz")
    for k, v in zip(("Pi", "S", "centroids", "boundaries"), host_constants(d)):
        assert np.array_equal(v, t[f"{k}_{d}"]), k


def test_reference_attend_f32_matches_reference_and_oracle(golden):
    """The timed CPU baseline (the reference's attend in its own precision)
    agrees with the reference-generated c0 output and with the fp64 oracle,
    single-threaded and on a thread pool alike."""
    A = golden("attend_c0.npz")
    c = CONFIGS["c0"]
    w = numpy_workload(100, c["B"], c["Hk"], c["Hq"], c["S"], c["D"], c["n_dec"])
    lay = O.compress_layer(w["k"], w["v"], dict(window_size=64))
    o1 = O.reference_attend_f32(lay, w["q"], threads=1)
    o4 = O.reference_attend_f32(lay, w["q"], threads=4)
    assert np.array_equal(o1, o4)
    assert np.abs(o1 - A["out"].reshape(o1.shape).astype(np.float32)).max() < 2e-3
    ref, _, _, _ = O.decode_attend(lay, w["q"])
    assert np.abs(o1 - ref).max() < 1e-5
    # with a decode buffer
    wd = numpy_workload(101, 2, 2, 8, 700, 128, 5)
    lay = O.compress_layer(wd["k"], wd["v"], dict(window_size=16))
    o = O.reference_attend_f32(lay, wd["q"], wd["dec_k"], wd["dec_v"], threads=2)
    ref, _, _, _ = O.decode_attend(lay, wd["q"], wd["dec_k"], wd["dec_v"])
    assert np.abs(o - ref).max() < 1e-5
