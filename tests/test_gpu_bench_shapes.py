"""GPU parity at the benchmarked shapes (configs c1, c2, c3 and c4).

Each benchmark line is only as good as the parity behind it, so the shapes the
bench measures are decoded here too and compared with the CPU oracle:

* c3 slice: B=2 of the 64 sequences, Hq32/Hk8, D128, S=32K, window 32, 10%
  near, with the benchmark's 1% injected spikes (keys 3 sigma along the
  group's mean query) at margin 0.5.  Every flag fires and every token is the
  earliest of the identical spike keys, so the tie-break is exercised too.
  The compressed tiers are checked bit for bit against the oracle first.
* c1 at S = 4K and 16K (G = 1, 32 KV heads; 9-13 splits per stream).
* c2: TurboQuant at S = 16K, Hq28/Hk4, with the planner's own split count
  (beyond the direct-load merge, i.e. the bulk-copy merge path).
* c4 long split: a 256K-token sequence, Hq32/Hk8, 5% near, split into 8
  equal-cost shards on one GPU (partial kernel per shard + combine), against
  the oracle's attention over the unsplit tiers.

Tolerances are the parity bar of the other decode tests (tests/helpers.py):
output max-abs 2e-3 and cosine 0.9999; flags and tokens identical.
"""

import numpy as np
import pytest
import torch

from oracle import fkv_oracle as O
from foveated_kv_b200 import TierConfig, compress_layer
from foveated_kv_b200.synthetic import numpy_workload, inject_spikes_np, CONFIGS
from foveated_kv_b200.turbo_constants import host_constants
from tests.helpers import np_, bits, layer_to_oracle, assert_output_close, assert_spikes_match

pytestmark = pytest.mark.gpu


def _cfg(name, **over):
    c = dict(CONFIGS[name])
    c.update(over)
    return c


def _tier_cfg(c, margin=0.5):
    return TierConfig(near_pct=c["near_pct"], n_sinks=c["n_sinks"], window_size=c["window_size"],
                      v_group=c["v_group"], compress_method=c["compress_method"],
                      select=c["select"], spike_margin=margin)


def _oracle_cfg(c):
    return dict(near_pct=c["near_pct"], n_sinks=c["n_sinks"], window_size=c["window_size"],
                v_group=c["v_group"], compress_method=c["compress_method"], select=c["select"])


@pytest.fixture(params=["tcgen05", "mma"])
def qk_path(request, monkeypatch):
    monkeypatch.setenv("FKV_QK_PATH", request.param)
    return request.param


@pytest.fixture(params=["tcgen05", "mma_cluster", "mma_flat"])
def launch_mode(request, monkeypatch):
    """q.K path and, on the mma.sync path, the cluster mode (CTAs of a
    stream share its stages dynamically and merge through distributed shared
    memory) or the flat split with workspace records (FKV_CLUSTER=0)."""
    path, _, flat = request.param.partition("_")
    monkeypatch.setenv("FKV_QK_PATH", "tcgen05" if path == "tcgen05" else "mma")
    monkeypatch.setenv("FKV_CLUSTER", "0" if flat == "flat" else "1")
    return request.param


def _plan(lay, Hq, turbo=False):
    import ctypes as C
    from foveated_kv_b200 import _native
    out = (C.c_int32 * 4)()
    sh = lay._fill_shape(Hq, lay.spike_margin)
    far = lay.far_k.data_ptr() if lay.far_k is not None and lay.far_k.numel() else None
    _native.check(_native.load().fkv_decode_plan(C.byref(sh), far, int(turbo), out), "plan")
    return list(out)


def _check_mode(lay, Hq, mode, turbo=False):
    nh, splits, csize, groups = _plan(lay, Hq, turbo)
    if mode == "tcgen05":
        assert nh > 0
    elif mode == "mma_cluster":
        assert nh == 0 and csize >= 2, (nh, splits, csize, groups)
    elif mode == "mma_flat":
        assert nh == 0 and csize == 0
    return nh, splits, csize, groups


def _decode_and_check(lay, w, margin, name, tc=None):
    t_q = torch.from_numpy(w["q"]).cuda()
    out, fl, tk = lay.attend_fused_with_spikes(t_q)
    torch.cuda.synchronize()
    rout, rfl, rtk, diag = O.decode_attend(layer_to_oracle(lay, tc), w["q"], None, None, margin)
    err, cos = assert_output_close(np_(out).astype(np.float64)[:, :, 0], rout, name)
    ties = assert_spikes_match(np_(fl), np_(tk), rfl, rtk, diag, margin, name)
    assert ties == 0, f"{name}: {ties} spike decisions within the tie band"
    return err, cos, np_(fl), np_(tk)


# ---- c3 slice with injected spikes ------------------------------------------------

@pytest.fixture(scope="module")
def c3_slice():
    c = _cfg("c3", B=2)
    w = numpy_workload(71, c["B"], c["Hk"], c["Hq"], c["S"], c["D"], 0)
    tb = O.tier_boundaries(c["S"], near_pct=c["near_pct"], n_sinks=c["n_sinks"],
                           window_size=c["window_size"])
    pos = inject_spikes_np(w, tb, 71)
    ref = O.compress_layer(w["k"], w["v"], _oracle_cfg(c))
    t = {k: torch.from_numpy(v).cuda() for k, v in w.items()}
    lay = compress_layer(t["k"], t["v"], _tier_cfg(c))
    torch.cuda.synchronize()
    del t
    return c, w, pos, ref, lay


def test_c3_slice_tiers_bit_exact(c3_slice):
    c, w, pos, ref, lay = c3_slice
    for f in ["near_k", "near_v", "near_idx", "near_valid", "far_idx", "far_k", "far_v",
              "far_v_scale", "far_v_zero", "archive_k", "archive_v"]:
        a, b = bits(np_(getattr(lay, f))), bits(ref[f])
        assert np.array_equal(a, b), f"c3 slice: {f} differs in {int((a != b).sum())} places"


def test_c3_slice_decode_with_spikes(c3_slice, qk_path):
    c, w, pos, ref, lay = c3_slice
    err, cos, fl, tk = _decode_and_check(lay, w, 0.5, f"c3 slice ({qk_path})")
    G = c["Hq"] // c["Hk"]
    assert fl.all(), "every head of the c3 slice holds forced spikes"
    # the spikes are identical keys: the token is the earliest spike position
    far0 = O.tier_boundaries(c["S"], near_pct=c["near_pct"], n_sinks=c["n_sinks"],
                             window_size=c["window_size"])["mid_start"]
    want = (pos.min(axis=2) - far0).repeat(G, axis=1)
    assert np.array_equal(tk, want)
    print(f"c3 slice {qk_path}: max-abs {err:.2e} cos {cos:.7f}")


# ---- c1 at 4K and 16K ----------------------------------------------------------------

@pytest.mark.parametrize("name", ["c1_4k", "c1_16k"])
def test_c1_decode(name, launch_mode):
    c = _cfg(name)
    w = numpy_workload(72, c["B"], c["Hk"], c["Hq"], c["S"], c["D"], 0)
    t = {k: torch.from_numpy(v).cuda() for k, v in w.items()}
    lay = compress_layer(t["k"], t["v"], _tier_cfg(c))
    plan = _check_mode(lay, c["Hq"], launch_mode)
    err, cos, _, _ = _decode_and_check(lay, w, 0.5, f"{name} ({launch_mode})")
    print(f"{name} {launch_mode} plan {plan}: max-abs {err:.2e} cos {cos:.7f}")


# ---- c2: TurboQuant at 16K ------------------------------------------------------------

@pytest.mark.parametrize("mode", ["cluster", "flat"])
def test_c2_turbo_decode_16k(mode, monkeypatch):
    monkeypatch.setenv("FKV_CLUSTER", "0" if mode == "flat" else "1")
    c = _cfg("c2")
    w = numpy_workload(73, c["B"], c["Hk"], c["Hq"], c["S"], c["D"], 0)
    t = {k: torch.from_numpy(v).cuda() for k, v in w.items()}
    lay = compress_layer(t["k"], t["v"], _tier_cfg(c))
    plan = _plan(lay, c["Hq"], turbo=True)
    assert (plan[2] >= 2) == (mode == "cluster"), plan
    pi, s, cen, bnd = host_constants(c["D"])
    tc = {"Pi": pi, "S": s, "centroids": cen, "boundaries": bnd}
    err, cos, _, _ = _decode_and_check(lay, w, 0.5, f"c2 turbo 16K ({mode})", tc)
    print(f"c2 {mode} plan {plan}: max-abs {err:.2e} cos {cos:.7f}")


# ---- c4: long sequence split into 8 shards on one GPU ------------------------------

@pytest.fixture(scope="module")
def c4_long():
    c = _cfg("c4", S=1 << 18)
    B, Hq, Hk, D, S = c["B"], c["Hq"], c["Hk"], c["D"], c["S"]
    w = numpy_workload(74, B, Hk, Hq, S, D, 0)
    tb = O.tier_boundaries(S, near_pct=c["near_pct"], n_sinks=c["n_sinks"],
                           window_size=c["window_size"])
    inject_spikes_np(w, tb, 74, frac=0.001)
    t = {k: torch.from_numpy(v).cuda() for k, v in w.items()}
    full = compress_layer(t["k"], t["v"], _tier_cfg(c), keep_archive=False)
    torch.cuda.synchronize()
    ref = O.decode_attend(layer_to_oracle(full), w["q"], None, None, 0.5)
    del full
    return c, t, ref


def test_c4_long_split_eight_shards(c4_long, qk_path):
    from foveated_kv_b200.seqsplit import shard_bounds_balanced, compress_shard, decode_partial, combine
    c, t, (rout, rfl, rtk, diag) = c4_long
    B, Hq, D, S = c["B"], c["Hq"], c["D"], c["S"]
    cfg = _tier_cfg(c)
    P = 8
    parts, args = [], []
    for r in range(P):
        lo, hi = shard_bounds_balanced(S, r, P, cfg)
        lay, off = compress_shard(t["k"][:, :, lo:hi], t["v"][:, :, lo:hi], S, lo, cfg)
        pa, ar = decode_partial(lay, t["q"], off)
        parts.append(pa.clone())
        args.append(ar.clone())
        del lay
    out, fl, tk = combine(torch.stack(parts), torch.stack(args), 0.5)
    torch.cuda.synchronize()
    err, cos = assert_output_close(np_(out).astype(np.float64).reshape(B, Hq, D), rout, "c4 split")
    ties = assert_spikes_match(np_(fl).reshape(B, Hq), np_(tk).reshape(B, Hq), rfl, rtk, diag,
                               0.5, "c4 split")
    assert ties == 0
    assert np_(fl).all()
    print(f"c4 256K split x{P} {qk_path}: max-abs {err:.2e} cos {cos:.7f}")


# ---- full-size properties (the oracle cannot finish these sizes quickly) -----------

def test_c3_full_batch_rows_match_slices():
    """c3 at its full size (B = 64, S = 32K, with the injected spikes): every
    sequence's outputs, flags and tokens from the 64-sequence launch equal
    those of the same sequence decoded in a 2-sequence launch (batch rows are
    independent), within the parity tolerance; the slices themselves are
    oracle-checked above."""
    from foveated_kv_b200.synthetic import torch_workload, inject_spikes_torch
    c = _cfg("c3")
    cfg = _tier_cfg(c)
    w = torch_workload(91, c["B"], c["Hk"], c["Hq"], c["S"], c["D"], 0, "cuda")
    inject_spikes_torch(w, cfg.tier_boundaries(c["S"]), 91)
    full = compress_layer(w["k"], w["v"], cfg, keep_archive=False)
    out, fl, tk = full.attend_fused_with_spikes(w["q"])
    out, fl, tk = out.clone(), fl.clone(), tk.clone()
    del full
    for b0 in (0, 30, 62):
        part = compress_layer(w["k"][b0:b0 + 2], w["v"][b0:b0 + 2], cfg, keep_archive=False)
        o2, f2, t2 = part.attend_fused_with_spikes(w["q"][b0:b0 + 2])
        torch.cuda.synchronize()
        err = (o2.float() - out[b0:b0 + 2].float()).abs().max().item()
        assert err <= 2e-3, (b0, err)
        assert torch.equal(f2, fl[b0:b0 + 2]) and torch.equal(t2, tk[b0:b0 + 2])
        del part
    assert bool(fl.all())


@pytest.mark.parametrize("P", [2, 8])
def test_c4_full_million_split_equals_unsplit(P):
    """c4 at its full length (S = 2^20, Hq32/Hk8, 5% near): the sequence split
    into P equal-cost shards on one GPU (partial kernel per shard + merge)
    equals the unsplit fused decode of the whole sequence within the parity
    tolerance, with identical flags and tokens (global far indices)."""
    from foveated_kv_b200.synthetic import torch_workload
    from foveated_kv_b200.seqsplit import shard_bounds_balanced, compress_shard, decode_partial, combine
    c = _cfg("c4")
    B, Hq, Hk, D, S = c["B"], c["Hq"], c["Hk"], c["D"], c["S"]
    cfg = _tier_cfg(c)
    w = torch_workload(92, B, Hk, Hq, S, D, 0, "cuda")
    full = compress_layer(w["k"], w["v"], cfg, keep_archive=False)
    ro, rf, rt = full.attend_fused_with_spikes(w["q"])
    ro, rf, rt = ro.clone(), rf.clone(), rt.clone()
    del full
    parts, args = [], []
    for r in range(P):
        lo, hi = shard_bounds_balanced(S, r, P, cfg)
        lay, off = compress_shard(w["k"][:, :, lo:hi], w["v"][:, :, lo:hi], S, lo, cfg)
        pa, ar = decode_partial(lay, w["q"], off)
        parts.append(pa.clone())
        args.append(ar.clone())
        del lay
    out, fl, tk = combine(torch.stack(parts), torch.stack(args), 0.5)
    torch.cuda.synchronize()
    err = (out.float() - ro.float().reshape(out.shape)).abs().max().item()
    assert err <= 2e-3, err
    assert torch.equal(fl, rf.reshape(-1)) and torch.equal(tk, rt.reshape(-1))
