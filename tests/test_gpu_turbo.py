"""GPU parity of the TurboQuant far tier: compression codes bit-exact vs the
oracle (fp64 restatement of turbo_quantize.py), and the fused decode kernel
scoring directly on codes vs the oracle's score-on-codes attention."""

import numpy as np
import pytest
import torch

from oracle import fkv_oracle as O
from foveated_kv_b200 import TierConfig, compress_layer
from foveated_kv_b200.turbo_constants import host_constants
from foveated_kv_b200.synthetic import numpy_workload
from tests.helpers import np_, bits, layer_to_oracle, assert_output_close, assert_spikes_match

pytestmark = pytest.mark.gpu


def _tc(D):
    pi, s, c, b = host_constants(D)
    return {"Pi": pi, "S": s, "centroids": c, "boundaries": b}


CASES = [
    # name, B, Hk, Hq, S, D, n_dec, cfg, margin
    ("c2_shape_4k", 1, 4, 28, 4096, 128, 0, dict(), 0.5),
    ("d64_b2", 2, 2, 8, 600, 64, 5, dict(), 0.5),
    ("g1_d128", 1, 3, 3, 900, 128, 17, dict(near_pct=0.2, window_size=8), 0.25),
]


@pytest.mark.parametrize("mode", ["cluster", "flat"])
@pytest.mark.parametrize("name,B,Hk,Hq,S,D,n_dec,kw,margin", CASES)
def test_turbo_compress_and_decode(name, B, Hk, Hq, S, D, n_dec, kw, margin, mode, monkeypatch):
    monkeypatch.setenv("FKV_CLUSTER", "0" if mode == "flat" else "1")
    w = numpy_workload(61, B, Hk, Hq, S, D, n_dec)
    t = {k: torch.from_numpy(v).cuda() for k, v in w.items()}
    cfg = TierConfig(compress_method="turbo", spike_margin=margin, **kw)
    lay = compress_layer(t["k"], t["v"], cfg)
    torch.cuda.synchronize()
    tc = _tc(D)
    ref = O.compress_layer(w["k"], w["v"], dict(compress_method="turbo", **kw), tc=tc)
    pairs = {"turbo_k_idx": lay.turbo_far_k_indices, "turbo_k_signs": lay.turbo_far_k_signs,
             "turbo_k_norm": lay.turbo_far_k_norm, "turbo_k_gamma": lay.turbo_far_k_gamma,
             "turbo_v_packed": lay.turbo_far_v_packed, "turbo_v_scale": lay.turbo_far_v_scale,
             "near_k": lay.near_k, "far_idx": lay.far_idx, "archive_k": lay.archive_k}
    for k, tv in pairs.items():
        a, b = bits(np_(tv)), bits(ref[k])
        assert np.array_equal(a, b), f"{name}: {k} differs in {int((a != b).sum())} places"
    for i in range(n_dec):
        lay.add_token(t["dec_k"][:, :, i:i + 1], t["dec_v"][:, :, i:i + 1])
    out, fl, tk = lay.attend_fused_with_spikes(t["q"])
    torch.cuda.synchronize()
    rout, rfl, rtk, diag = O.decode_attend(layer_to_oracle(lay, tc), w["q"], w["dec_k"],
                                           w["dec_v"], margin)
    assert_output_close(np_(out).astype(np.float64)[:, :, 0], rout, name)
    assert assert_spikes_match(np_(fl), np_(tk), rfl, rtk, diag, margin, name) == 0
