"""GPU parity: fp8/INT4 compression and the fused decode kernel vs the CPU
oracle, through libfkv.so's C ABI (via the package surface)."""

import ctypes as C

import numpy as np
import pytest
import torch

from oracle import fkv_oracle as O
from foveated_kv_b200 import TierConfig, compress_layer, _native
from foveated_kv_b200.synthetic import numpy_workload, CONFIGS
from tests.helpers import (np_, bits, layer_to_oracle, assert_output_close,
                           assert_spikes_match)

pytestmark = pytest.mark.gpu

dev = "cuda"


def _tensors(w):
    return {k: torch.from_numpy(v).to(dev) for k, v in w.items()}


def _cfg_dict(cfg: TierConfig):
    return dict(near_pct=cfg.near_pct, n_sinks=cfg.n_sinks, window_size=cfg.window_size,
                promo_headroom_pct=cfg.promo_headroom_pct,
                promo_headroom_min=cfg.promo_headroom_min, compress_method=cfg.compress_method,
                select=cfg.select, v_group=cfg.v_group)


COMPRESS_CASES = [
    # name, B, Hk, Hq, S, D, cfg kwargs
    ("c0_recency", 1, 2, 14, 1024, 64, dict(window_size=64)),
    ("c0_vg32", 1, 2, 14, 1024, 64, dict(window_size=64, v_group=32)),
    ("c1_1k", 1, 32, 32, 1024, 128, dict(window_size=128)),
    ("b3_d128_vg32", 3, 2, 8, 300, 128, dict(window_size=16, v_group=32, near_pct=0.2)),
    ("tiny_no_far", 1, 1, 1, 20, 64, dict()),
    ("S1", 2, 1, 4, 1, 64, dict()),
]


@pytest.mark.parametrize("name,B,Hk,Hq,S,D,kw", COMPRESS_CASES)
def test_compress_fp8_bit_exact(name, B, Hk, Hq, S, D, kw):
    w = numpy_workload(11, B, Hk, Hq, S, D, 0)
    cfg = TierConfig(**kw)
    ref = O.compress_layer(w["k"], w["v"], _cfg_dict(cfg))
    t = _tensors(w)
    lay = compress_layer(t["k"], t["v"], cfg)
    torch.cuda.synchronize()
    pairs = {"near_k": lay.near_k, "near_v": lay.near_v, "near_idx": lay.near_idx,
             "near_valid": lay.near_valid, "far_idx": lay.far_idx, "far_k": lay.far_k,
             "far_v": lay.far_v, "far_v_scale": lay.far_v_scale, "far_v_zero": lay.far_v_zero,
             "archive_k": lay.archive_k, "archive_v": lay.archive_v}
    for k, tv in pairs.items():
        a, b = bits(np_(tv)), bits(ref[k])
        assert a.shape == b.shape, (k, a.shape, b.shape)
        assert np.array_equal(a, b), f"{name}: {k} differs at {np.argwhere(a != b)[:5]}"


def test_compress_golden_c0_layer(golden):
    """Device compression reproduces the reference-generated c0 layer fixture."""
    L = golden("layer_c0_fp8.npz")
    c = CONFIGS["c0"]
    w = numpy_workload(100, c["B"], c["Hk"], c["Hq"], c["S"], c["D"], c["n_dec"])
    t = _tensors(w)
    lay = compress_layer(t["k"], t["v"], TierConfig(window_size=64))
    for f in ["near_k", "near_v", "near_idx", "far_k", "far_v", "far_v_scale", "far_v_zero",
              "far_idx", "archive_k", "archive_v"]:
        assert np.array_equal(bits(np_(getattr(lay, f))), bits(L[f])), f
    assert np.all(np_(lay.near_valid) == L["near_valid"][None])


DECODE_CASES = [
    # name, B, Hk, Hq, S, D, n_dec, cfg kwargs, margin
    ("c0_shape_dec16", 1, 2, 14, 1024, 64, 16, dict(window_size=64), 0.5),
    ("c0_vg32", 1, 2, 14, 1024, 64, 16, dict(window_size=64, v_group=32), 0.5),
    ("c1_1k_g1", 1, 32, 32, 1024, 128, 0, dict(window_size=128), 0.5),
    ("g4_b2", 2, 4, 16, 2048, 128, 5, dict(), 0.5),
    ("g8_d128", 1, 2, 16, 3000, 128, 33, dict(v_group=32), 1.0),
    ("g16_two_head_groups", 1, 1, 16, 700, 64, 3, dict(), 0.5),
    ("g3_ragged", 3, 3, 9, 517, 128, 7, dict(near_pct=0.25, window_size=8), 0.25),
    ("no_far", 1, 2, 4, 30, 64, 4, dict(near_pct=0.9), 0.5),
]


@pytest.fixture(params=["tcgen05", "mma", "mma_flat"])
def qk_path(request, monkeypatch):
    """Run a decode test on each far-tier q.K path: tcgen05 (tensor memory,
    forced with FKV_QK_PATH=tcgen05 where the shape allows it) and mma.sync
    (FKV_QK_PATH=mma).  The default picks one per shape by CTA work size.
    On the mma.sync path small shapes run in cluster mode (the CTAs of a
    stream share its stages and merge through distributed shared memory);
    mma_flat turns it off (FKV_CLUSTER=0: split records in the workspace)."""
    monkeypatch.setenv("FKV_QK_PATH", "tcgen05" if request.param == "tcgen05" else "mma")
    monkeypatch.setenv("FKV_CLUSTER", "0" if request.param == "mma_flat" else "1")
    return request.param


def _expect_path(lay, Hq, path):
    """The library reports the q.K path the launch takes: tcgen05 (4 or 8 q
    heads per CTA) for D = 128 with a far tier when forced, else mma.sync."""
    lib = _native.load()
    sh = lay._fill_shape(Hq, lay.spike_margin)
    got = lib.fkv_decode_qk_path(C.byref(sh), lay.far_k.data_ptr())
    G = Hq // lay.near_k.shape[1]
    want_tc = path == "tcgen05" and lay.near_k.shape[-1] == 128 and lay.n_far > 0
    assert (got > 0) == want_tc, (got, path, G)
    if want_tc:
        assert got == (4 if G <= 4 else 8)


@pytest.mark.parametrize("name,B,Hk,Hq,S,D,n_dec,kw,margin", DECODE_CASES)
def test_decode_fp8_parity(name, B, Hk, Hq, S, D, n_dec, kw, margin, qk_path):
    w = numpy_workload(23, B, Hk, Hq, S, D, n_dec)
    cfg = TierConfig(spike_margin=margin, **kw)
    t = _tensors(w)
    lay = compress_layer(t["k"], t["v"], cfg)
    _expect_path(lay, Hq, qk_path)
    for i in range(n_dec):
        lay.add_token(t["dec_k"][:, :, i:i + 1], t["dec_v"][:, :, i:i + 1])
    out, flags, tokens = lay.attend_fused_with_spikes(t["q"][:, :, None, :])
    torch.cuda.synchronize()
    ref_lay = layer_to_oracle(lay)
    rout, rflags, rtok, diag = O.decode_attend(ref_lay, w["q"], w["dec_k"], w["dec_v"], margin)
    assert_output_close(np_(out).astype(np.float64)[:, :, 0], rout, name)
    ties = assert_spikes_match(np_(flags), np_(tokens), rflags, rtok, diag, margin, name)
    assert ties == 0


@pytest.mark.parametrize("splits", [1, 2, 3, 7, 40])
def test_decode_split_counts_agree(splits, qk_path):
    """Explicit split counts through the raw C ABI give the same answer."""
    w = numpy_workload(5, 2, 2, 8, 1500, 128, 9)
    t = _tensors(w)
    lay = compress_layer(t["k"], t["v"], TierConfig())
    for i in range(9):
        lay.add_token(t["dec_k"][:, :, i:i + 1], t["dec_v"][:, :, i:i + 1])
    lib = _native.load()
    sh = _native.DecodeShape(B=2, Hq=8, Hk=2, D=128, n_near_alloc=lay.n_near_alloc,
                             n_far=lay.n_far, n_dec=9, dec_stride=lay._dec_k.shape[2], v_group=0,
                             num_splits=splits, spike_margin=0.5)
    ws = torch.zeros(lib.fkv_decode_workspace_bytes(C.byref(sh)) + 16, dtype=torch.uint8,
                     device=dev)
    out = torch.empty((2, 8, 128), dtype=torch.float16, device=dev)
    fl = torch.empty((2, 8), dtype=torch.int32, device=dev)
    tk = torch.empty_like(fl)
    p = lambda x: x.data_ptr()
    for rep in range(2):   # second call reuses the workspace (counters back at zero)
        rc = lib.fkv_decode_fp8(C.byref(sh), p(lay.near_k), p(lay.near_v), p(lay.near_valid),
                                p(lay.far_k), p(lay.far_v), p(lay.far_v_scale),
                                p(lay.far_v_zero), p(t["q"]), p(lay._dec_k), p(lay._dec_v),
                                p(out), p(fl), p(tk), p(ws), ws.numel(),
                                torch.cuda.current_stream().cuda_stream)
        _native.check(rc, "fkv_decode_fp8")
        torch.cuda.synchronize()
        rout, rfl, rtk, diag = O.decode_attend(layer_to_oracle(lay), w["q"], w["dec_k"],
                                               w["dec_v"], 0.5)
        assert_output_close(np_(out).astype(np.float64), rout, f"splits={splits}")
        assert assert_spikes_match(np_(fl), np_(tk), rfl, rtk, diag, 0.5) == 0


def test_decode_per_head_near_valid():
    """Promoted rows in headroom are attended only up to near_valid[b, h]."""
    w = numpy_workload(9, 2, 2, 8, 800, 64, 0)
    t = _tensors(w)
    lay = compress_layer(t["k"], t["v"], TierConfig(spike_margin=0.5))
    R = int(lay.near_valid[0, 0])
    # write 3 archive rows of (b=0,h=1) and 1 row of (b=1,h=0) into headroom
    lay.near_k[0, 1, R:R + 3] = lay.archive_k[0, 1, 10:13]
    lay.near_v[0, 1, R:R + 3] = lay.archive_v[0, 1, 10:13]
    lay.near_valid[0, 1] += 3
    lay.near_k[1, 0, R] = lay.archive_k[1, 0, 0]
    lay.near_v[1, 0, R] = lay.archive_v[1, 0, 0]
    lay.near_valid[1, 0] += 1
    out, fl, tk = lay.attend_fused_with_spikes(t["q"])
    torch.cuda.synchronize()
    rout, rfl, rtk, diag = O.decode_attend(layer_to_oracle(lay), w["q"], None, None, 0.5)
    assert_output_close(np_(out).astype(np.float64)[:, :, 0], rout, "near_valid")
    assert assert_spikes_match(np_(fl), np_(tk), rfl, rtk, diag, 0.5) == 0


def test_decode_buffer_growth_and_flags_all_set():
    """Decode buffer beyond its first capacity; margin -inf-like forces flags."""
    w = numpy_workload(3, 1, 2, 4, 400, 128, 40)
    t = _tensors(w)
    lay = compress_layer(t["k"], t["v"], TierConfig(spike_margin=-1e4))
    for i in range(40):
        lay.add_token(t["dec_k"][:, :, i:i + 1], t["dec_v"][:, :, i:i + 1])
    out, fl, tk = lay.attend_fused_with_spikes(t["q"])
    torch.cuda.synchronize()
    assert np.all(np_(fl) == 1)
    rout, rfl, rtk, diag = O.decode_attend(layer_to_oracle(lay), w["q"], w["dec_k"], w["dec_v"],
                                           -1e4)
    assert_output_close(np_(out).astype(np.float64)[:, :, 0], rout, "dec40")
    assert np.array_equal(np_(tk), rtk)


def _raw_decode(lay, sh, q, Hq, D):
    """fkv_decode_fp8 through the C ABI with the shape as given (twice: the
    second call reuses the workspace, whose counters the first put back)."""
    lib = _native.load()
    B = q.shape[0]
    ws = torch.zeros(lib.fkv_decode_workspace_bytes(C.byref(sh)) + 16, dtype=torch.uint8,
                     device=dev)
    out = torch.empty((B, Hq, D), dtype=torch.float16, device=dev)
    fl = torch.empty((B, Hq), dtype=torch.int32, device=dev)
    tk = torch.empty_like(fl)
    p = lambda x: x.data_ptr()
    for _ in range(2):
        rc = lib.fkv_decode_fp8(C.byref(sh), p(lay.near_k), p(lay.near_v), p(lay.near_valid),
                                p(lay.far_k), p(lay.far_v), p(lay.far_v_scale),
                                p(lay.far_v_zero), p(q), p(lay._dec_k), p(lay._dec_v),
                                p(out), p(fl), p(tk), p(ws), ws.numel(),
                                torch.cuda.current_stream().cuda_stream)
        _native.check(rc, "fkv_decode_fp8")
    torch.cuda.synchronize()
    return out, fl, tk


@pytest.mark.parametrize("G,D,splits", [(1, 128, 13), (1, 128, 32), (1, 128, 48), (2, 128, 16), (1, 64, 60), (2, 64, 60),
                                         (4, 64, 16)])
def test_decode_few_heads_many_splits(G, D, splits, qk_path):
    """Streams with few q heads (G < 8) and more split records than the direct
    merge takes: the last CTA merges only the active heads' outputs, spread
    over thread groups that each take every k-th record."""
    Hk, S = 2, 4000
    w = numpy_workload(11, 1, Hk, G * Hk, S, D, 3)
    t = _tensors(w)
    lay = compress_layer(t["k"], t["v"], TierConfig())
    for i in range(3):
        lay.add_token(t["dec_k"][:, :, i:i + 1], t["dec_v"][:, :, i:i + 1])
    sh = lay._fill_shape(G * Hk, 0.5)
    sh.num_splits = splits
    out, fl, tk = _raw_decode(lay, sh, t["q"], G * Hk, D)
    rout, rfl, rtk, diag = O.decode_attend(layer_to_oracle(lay), w["q"], w["dec_k"], w["dec_v"], 0.5)
    assert_output_close(np_(out).astype(np.float64), rout, f"G={G} D={D} splits={splits}")
    assert assert_spikes_match(np_(fl), np_(tk), rfl, rtk, diag, 0.5) == 0


@pytest.mark.parametrize("splits", [1, 0])
def test_decode_long_stream_accumulation(splits, qk_path):
    """One 32K-token stream decoded by as few CTAs as possible (splits=1): the
    longest per-warp accumulation of P.V, which stresses the f32 accumulator
    (raw INT4 codes enter the product with their magic-number offsets, removed
    once per warp record)."""
    S, B, Hk, Hq, D = 32768, 1, 1, 4, 128
    w = numpy_workload(31, B, Hk, Hq, S, D, 0)
    t = _tensors(w)
    lay = compress_layer(t["k"], t["v"], TierConfig(spike_margin=0.5))
    lib = _native.load()
    sh = lay._fill_shape(Hq, 0.5)
    sh.num_splits = splits
    ws = torch.zeros(lib.fkv_decode_workspace_bytes(C.byref(sh)) + 16, dtype=torch.uint8,
                     device=dev)
    out = torch.empty((B, Hq, D), dtype=torch.float16, device=dev)
    fl = torch.empty((B, Hq), dtype=torch.int32, device=dev)
    tk = torch.empty_like(fl)
    p = lambda x: x.data_ptr()
    rc = lib.fkv_decode_fp8(C.byref(sh), p(lay.near_k), p(lay.near_v), p(lay.near_valid),
                            p(lay.far_k), p(lay.far_v), p(lay.far_v_scale), p(lay.far_v_zero),
                            p(t["q"]), 0, 0, p(out), p(fl), p(tk), p(ws), ws.numel(),
                            torch.cuda.current_stream().cuda_stream)
    _native.check(rc, "fkv_decode_fp8")
    torch.cuda.synchronize()
    rout, rfl, rtk, diag = O.decode_attend(layer_to_oracle(lay), w["q"], None, None, 0.5)
    err, cos = assert_output_close(np_(out).astype(np.float64), rout, f"long splits={splits}")
    print(f"long stream splits={splits} path={qk_path}: max-abs {err:.2e} cos {cos:.7f}")
    assert assert_spikes_match(np_(fl), np_(tk), rfl, rtk, diag, 0.5) == 0


def test_compress_int4_rounding_boundaries():
    """V rows built so that (v - min) / scale lands exactly on, or next to,
    the half-integer rounding boundaries of the INT4 codes (where the kernel
    falls back from the reciprocal product to the correctly rounded division):
    codes must still equal the oracle's bit for bit."""
    rng = np.random.default_rng(3)
    B, H, S, D = 1, 2, 400, 128
    w = numpy_workload(41, B, H, 4, S, D, 0)
    v = w["v"].copy()
    for h in range(H):
        for s in range(S):
            kind = s % 4
            k = rng.integers(0, 15, D).astype(np.float64)
            if kind == 0:      # scale 1: exact ties k + 0.5
                row = k + 0.5
                row[0], row[1] = 0.0, 15.0
            elif kind == 1:    # scale 0.5, min -3: exact ties
                row = -3.0 + 0.5 * (k + 0.5)
                row[0], row[1] = -3.0, 4.5
            elif kind == 2:    # scale 1/15 (inexact): fp16 values next to the ties
                row = (k + 0.5) / 15.0
                row[0], row[1] = 0.0, 1.0
            else:              # ordinary data
                continue
            v[0, h, s] = row.astype(np.float16)
    w["v"] = v
    cfg = TierConfig(window_size=16)
    ref = O.compress_layer(w["k"], w["v"], _cfg_dict(cfg))
    t = _tensors(w)
    lay = compress_layer(t["k"], t["v"], cfg)
    torch.cuda.synchronize()
    for f in ["far_v", "far_v_scale", "far_v_zero", "far_k"]:
        a, b = bits(np_(getattr(lay, f))), bits(ref[f])
        assert np.array_equal(a, b), f"{f} differs at {np.argwhere(a != b)[:5]}"


def test_compress_fp8_all_fp16_patterns():
    """Every one of the 65,536 fp16 bit patterns (zeros, subnormals, the
    underflow and overflow boundaries, inf, NaN) goes through the device fp8
    encoder as far-tier K and must give the oracle's E4M3 code (the
    reference's _fp16_to_e4m3 semantics, pinned by the golden table)."""
    S, D = 600, 128
    w = numpy_workload(5, 1, 1, 1, S, D, 0)
    pats = np.arange(65536, dtype=np.uint32).astype(np.uint16).view(np.float16).reshape(512, D)
    k = w["k"].copy()
    k[0, 0, 4:4 + 512] = pats
    cfg = TierConfig(near_pct=0.0, window_size=8)
    t = _tensors({"k": k, "v": w["v"]})
    lay = compress_layer(t["k"], t["v"], cfg)
    torch.cuda.synchronize()
    far_idx = np_(lay.far_idx)[0, 0]
    assert far_idx[0] == 4 and np.all(np.diff(far_idx) == 1)
    got = np_(lay.far_k)[0, 0, :512].reshape(-1)
    want = O.fp16_to_e4m3(pats.reshape(-1))
    bad = np.argwhere(got != want).reshape(-1)
    assert bad.size == 0, [(hex(int(pats.reshape(-1).view(np.uint16)[i])), hex(int(got[i])), hex(int(want[i]))) for i in bad[:8]]
