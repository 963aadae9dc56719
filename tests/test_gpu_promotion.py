"""GPU: promotion of exact fp16 rows into near headroom through the C++
worker, the stream-ordered near_valid bump, and decode parity afterwards."""

import numpy as np
import pytest
import torch

from oracle import fkv_oracle as O
from foveated_kv_b200 import TierConfig, compress_layer, PromotionPipeline
from foveated_kv_b200.synthetic import numpy_workload
from tests.helpers import np_, bits, layer_to_oracle, assert_output_close, assert_spikes_match

pytestmark = pytest.mark.gpu


def _setup(B=2, Hk=2, Hq=8, S=600, D=128, margin=0.5, headroom_min=8):
    w = numpy_workload(41, B, Hk, Hq, S, D, 0)
    t = {k: torch.from_numpy(v).cuda() for k, v in w.items()}
    cfg = TierConfig(spike_margin=margin, promo_headroom_pct=0.0, promo_headroom_min=headroom_min)
    return w, t, compress_layer(t["k"], t["v"], cfg)


def test_promotion_closed_loop_and_parity():
    w, t, lay = _setup()
    pipe = PromotionPipeline(1, cooldown_steps=0, max_per_drain=64)
    pipe.register_archive_host(0, lay.archive_k.cpu().pin_memory(), lay.archive_v.cpu().pin_memory(),
                               lay.far_idx)
    pipe.register_blob(0, lay.get_blob_info())
    R0 = np_(lay.near_valid).copy()
    promoted = {}
    for step in range(3):
        out, fl, tk = lay.attend_fused_with_spikes(t["q"])
        fl_h, tk_h = np_(fl), np_(tk)
        n = pipe.drain_spikes(0, fl_h, tk_h, lay.far_idx, step)
        pipe.flush()
        torch.cuda.synchronize()
        G = 4
        seen = set()
        for b in range(2):
            for hq in range(8):
                if fl_h[b, hq] and (b, hq // G) not in seen:
                    seen.add((b, hq // G))
                    promoted.setdefault((b, hq // G), []).append(int(tk_h[b, hq]))
        assert n >= 0
    nv = np_(lay.near_valid)
    st = pipe.get_stats()
    assert st["promotions_completed"] == int((nv - R0).sum()) > 0
    # promoted rows are the exact archive rows, in promotion order
    arc_k, near_k = np_(lay.archive_k), np_(lay.near_k)
    for (b, h), toks in promoted.items():
        uniq = list(dict.fromkeys(toks))
        for j, fl_ in enumerate(uniq[: nv[b, h] - R0[b, h]]):
            assert np.array_equal(bits(near_k[b, h, R0[b, h] + j]), bits(arc_k[b, h, fl_]))
    # decode over the grown near tier matches the oracle (promoted rows attended twice)
    out, fl, tk = lay.attend_fused_with_spikes(t["q"])
    torch.cuda.synchronize()
    rout, rfl, rtk, diag = O.decode_attend(layer_to_oracle(lay), w["q"], None, None, 0.5)
    assert_output_close(np_(out).astype(np.float64)[:, :, 0], rout, "after promotion")
    assert assert_spikes_match(np_(fl), np_(tk), rfl, rtk, diag, 0.5) == 0
    pipe.close()


def test_headroom_full_is_counted():
    w, t, lay = _setup(B=1, Hk=1, Hq=4, headroom_min=2)
    pipe = PromotionPipeline(1, cooldown_steps=0, max_per_drain=8)
    pipe.register_archive_host(0, lay.archive_k.cpu(), lay.archive_v.cpu(), lay.far_idx)
    pipe.register_blob(0, lay.get_blob_info())
    R = int(lay.near_valid[0, 0])
    for step in range(5):   # 5 distinct far tokens, only 2 headroom slots
        pipe.drain_spikes(0, np.array([[1, 0, 0, 0]], np.int32), np.array([[step, 0, 0, 0]], np.int32),
                          lay.far_idx, step)
    pipe.flush()
    torch.cuda.synchronize()
    st = pipe.get_stats()
    assert st["promotions_completed"] == 2 and st["promotions_headroom_full"] == 3
    assert int(lay.near_valid[0, 0]) == R + 2
    pipe.close()


def test_promotion_from_disk_archive_bit_exact(tmp_path):
    """Rows promoted from an mmapped on-disk archive (the reference's
    archive_{k,v}_layer{L}.bin format, disk_archive.py:127-185) land in the
    device near tier bit for bit (promotion_pipeline.cpp:45-83,225-233)."""
    from foveated_kv_b200 import create_disk_archive
    w, t, lay = _setup(B=2, Hk=2, Hq=8)
    arc = create_disk_archive(lay.archive_k, lay.archive_v, lay.far_idx, 0, tmp_path)
    B, Hk, F, D = lay.archive_k.shape
    pipe = PromotionPipeline(1, cooldown_steps=0, max_per_drain=64)
    pipe.register_archive(0, arc.path_k, arc.path_v, Hk, F, D, lay.far_idx, B=B)
    pipe.register_blob(0, lay.get_blob_info())
    R0 = np_(lay.near_valid).copy()
    # flag every q head; the first head of each (b, kv head) names a far token
    toks = np.array([[3, 0, 0, 0, 17, 0, 0, 0], [5, 0, 0, 0, 40, 0, 0, 0]], np.int32)
    n = pipe.drain_spikes(0, np.ones((2, 8), np.int32), toks, lay.far_idx, 0)
    assert n == 4
    pipe.flush()
    torch.cuda.synchronize()
    nv = np_(lay.near_valid)
    assert np.array_equal(nv - R0, np.ones((2, 2), np.int32))
    near_k, near_v = np_(lay.near_k), np_(lay.near_v)
    for b in range(2):
        for h in range(2):
            fl_ = toks[b, 4 * h]
            assert np.array_equal(bits(near_k[b, h, R0[b, h]]), bits(np.array(arc.mmap_k[b, h, fl_])))
            assert np.array_equal(bits(near_v[b, h, R0[b, h]]), bits(np.array(arc.mmap_v[b, h, fl_])))
    assert pipe.get_stats()["promotions_completed"] == 4
    pipe.close()
    arc.close()


def test_large_batched_promotion_matches_archive():
    """Hundreds of rows queued across drains move in batches (one H2D copy of
    packed rows per batch, a scatter kernel, then the counts); every row is
    exact and near_valid counts every row."""
    B, Hk, Hq, S, D = 8, 8, 32, 2000, 128
    w = numpy_workload(43, B, Hk, Hq, S, D, 0)
    t = {k: torch.from_numpy(v).cuda() for k, v in w.items()}
    lay = compress_layer(t["k"], t["v"], TierConfig(spike_margin=0.5))
    pipe = PromotionPipeline(1, cooldown_steps=0, max_per_drain=10000)
    pipe.register_archive_host(0, lay.archive_k.cpu().pin_memory(), lay.archive_v.cpu().pin_memory(),
                               lay.far_idx)
    pipe.register_blob(0, lay.get_blob_info())
    R0 = np_(lay.near_valid).copy()
    rng = np.random.default_rng(0)
    picks = {}
    for step in range(6):      # 64 streams x 6 steps, position-deduplicated
        toks = rng.integers(0, lay.n_far, (B, Hq)).astype(np.int32)
        pipe.drain_spikes(0, np.ones((B, Hq), np.int32), toks, lay.far_idx, step)
        for b in range(B):
            for h in range(Hk):
                picks.setdefault((b, h), [])
                if toks[b, 4 * h] not in picks[(b, h)]:
                    picks[(b, h)].append(int(toks[b, 4 * h]))
    pipe.flush()
    torch.cuda.synchronize()
    nv = np_(lay.near_valid)
    near_k, near_v = np_(lay.near_k), np_(lay.near_v)
    arc_k, arc_v = np_(lay.archive_k), np_(lay.archive_v)
    total = 0
    for (b, h), toks in picks.items():
        assert nv[b, h] - R0[b, h] == len(toks)
        for j, fl_ in enumerate(toks):
            assert np.array_equal(bits(near_k[b, h, R0[b, h] + j]), bits(arc_k[b, h, fl_]))
            assert np.array_equal(bits(near_v[b, h, R0[b, h] + j]), bits(arc_v[b, h, fl_]))
        total += len(toks)
    assert pipe.get_stats()["promotions_completed"] == total
    pipe.close()


def test_async_promotion_then_parity():
    """Promotions left to the worker between steps (no flush: the
    reference's default asynchronous mode) overlap the next decodes; every
    launch reads a snapshot of near_valid, and after a final flush the tiers
    and the decode agree with the oracle."""
    w, t, lay = _setup(B=2, Hk=2, Hq=8, S=1500)
    pipe = PromotionPipeline(1, cooldown_steps=0, max_per_drain=64)
    pipe.register_archive_host(0, lay.archive_k.cpu().pin_memory(), lay.archive_v.cpu().pin_memory(),
                               lay.far_idx)
    pipe.register_blob(0, lay.get_blob_info())
    R0 = np_(lay.near_valid).copy()
    rng = np.random.default_rng(1)
    for step in range(6):
        out, fl, tk = lay.attend_fused_with_spikes(t["q"])
        toks = rng.integers(0, lay.n_far, (2, 8)).astype(np.int32)
        pipe.drain_spikes(0, np.ones((2, 8), np.int32), toks, lay.far_idx, step)
        assert torch.isfinite(out.float()).all()
    pipe.flush()
    torch.cuda.synchronize()
    nv = np_(lay.near_valid)
    assert int((nv - R0).sum()) == pipe.get_stats()["promotions_completed"] > 0
    out, fl, tk = lay.attend_fused_with_spikes(t["q"])
    torch.cuda.synchronize()
    rout, rfl, rtk, diag = O.decode_attend(layer_to_oracle(lay), w["q"], None, None, 0.5)
    assert_output_close(np_(out).astype(np.float64)[:, :, 0], rout, "after async promotion")
    pipe.close()
