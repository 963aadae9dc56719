"""GPU: importance-ranked tier selection vs the oracle's specification
(fp64 softmax mass summed over the GQA group; sinks + window always near;
ties to the lower position), then the full compression bit-exact."""

import numpy as np
import pytest
import torch

from oracle import fkv_oracle as O
from foveated_kv_b200 import TierConfig, compress_layer
from foveated_kv_b200.synthetic import numpy_workload, CONFIGS
from tests.helpers import np_, bits

pytestmark = pytest.mark.gpu

CASES = [
    ("c0", 1, 2, 14, 1024, 64, dict(window_size=64, v_group=32)),
    ("g1_d128", 2, 3, 3, 2000, 128, dict(window_size=16)),
    ("g4_b2", 2, 2, 8, 777, 128, dict(near_pct=0.3)),
    ("ties", 1, 2, 4, 300, 64, dict(near_pct=0.2, window_size=8)),
    ("all_middle_near", 1, 1, 2, 50, 64, dict(near_pct=1.0, window_size=4)),
]


@pytest.mark.parametrize("name,B,Hk,Hq,S,D,kw", CASES)
def test_importance_compress_bit_exact(name, B, Hk, Hq, S, D, kw):
    w = numpy_workload(71, B, Hk, Hq, S, D, 0)
    if name == "ties":
        w["k"][:, :, 50:250] = 0      # 200 exactly-tied middle tokens
    t = {k: torch.from_numpy(v).cuda() for k, v in w.items()}
    cfg = TierConfig(select="importance", **kw)
    lay = compress_layer(t["k"], t["v"], cfg, query=t["q_obs"])
    torch.cuda.synchronize()
    ref = O.compress_layer(w["k"], w["v"], dict(select="importance", **kw), q_obs=w["q_obs"])
    for f in ["near_idx", "far_idx", "near_valid", "near_k", "near_v", "far_k", "far_v",
              "far_v_scale", "far_v_zero", "archive_k"]:
        a, b = bits(np_(getattr(lay, f))), bits(ref[f])
        assert a.shape == b.shape, (f, a.shape, b.shape)
        assert np.array_equal(a, b), f"{name}: {f} differs at {np.argwhere(a != b)[:4]}"
