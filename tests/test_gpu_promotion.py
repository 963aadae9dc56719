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
