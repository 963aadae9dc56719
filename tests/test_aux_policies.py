"""Auxiliary host policies around the hot path: GQA-mean ``detect_spikes``
(mlx_foveated.py:451-490), archive rescoring (disk_archive.py:89-109) on CPU,
and per-layer compression on a side stream overlapping prefill (GPU)."""

import math

import numpy as np
import pytest
import torch

from oracle import fkv_oracle as O
from foveated_kv_b200 import FoveatedLayer, FoveatedKVCache, TierConfig, create_disk_archive
from foveated_kv_b200.synthetic import numpy_workload


def _cpu_layer(w, cfg):
    lay = O.compress_layer(w["k"], w["v"], cfg)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a))
    return lay, FoveatedLayer(near_k=t(lay["near_k"]), near_v=t(lay["near_v"]),
                              near_idx=t(lay["near_idx"]), near_valid=t(lay["near_valid"]),
                              far_idx=t(lay["far_idx"]), far_k=t(lay["far_k"]),
                              far_v=t(lay["far_v"]), far_v_scale=t(lay["far_v_scale"]),
                              far_v_zero=t(lay["far_v_zero"]))


@pytest.mark.gpu
@pytest.mark.parametrize("margin", [-100.0, 0.5, 2.0, 1e6])
def test_detect_spikes_matches_reference_semantics(margin):
    """detect_spikes runs as one fused launch with the GQA-mean query; it
    equals a restatement of mlx_foveated.py:451-490 (near + decode scores,
    far E4M3 scores, 1/sqrt(D)) on the same tiers."""
    from foveated_kv_b200 import compress_layer
    w = numpy_workload(3, 2, 2, 8, 1400, 128, 3)
    t = {k: torch.from_numpy(v).cuda() for k, v in w.items()}
    lay = compress_layer(t["k"], t["v"], TierConfig(near_pct=0.1, window_size=16))
    for j in range(3):
        lay.add_token(t["dec_k"][:, :, j:j + 1], t["dec_v"][:, :, j:j + 1])
    got = lay.detect_spikes(t["q"], margin)
    q = w["q"].astype(np.float32).reshape(2, 2, 4, 128).mean(2).astype(np.float16).astype(np.float64)
    rows, near_v = [], lay.near_valid.cpu().numpy()
    nk, fk = lay.near_k.cpu().numpy(), lay.far_k.cpu().numpy()
    for b in range(2):
        for h in range(2):
            keys = np.concatenate([nk[b, h, :near_v[b, h]], w["dec_k"][b, h]]).astype(np.float64)
            ns = keys @ q[b, h] / math.sqrt(128)
            fs = O.e4m3_to_fp16(fk[b, h]).astype(np.float64) @ q[b, h] / math.sqrt(128)
            gap = fs.max() - (ns.min() + margin)
            assert abs(gap) > 1e-3, "seeded case sits on the decision"
            if gap > 0:
                rows.append([b, h, int(np.argmax(fs))])
    if not rows:
        assert got is None
    else:
        assert np.array_equal(got.cpu().numpy(), np.array(rows, dtype=np.int32))


def test_fused_calls_reject_host_tensors():
    w = numpy_workload(3, 1, 2, 8, 400, 64, 0)
    lay, fl = _cpu_layer(w, dict(near_pct=0.1, window_size=16))
    with pytest.raises(ValueError, match="CUDA"):
        fl.attend_fused_with_spikes(torch.from_numpy(w["q"]))


def test_archive_rescoring(tmp_path):
    rs = np.random.RandomState(0)
    k = rs.standard_normal((1, 2, 20, 16)).astype(np.float16)
    arc = create_disk_archive(torch.from_numpy(k), torch.from_numpy(k), torch.zeros(1, 2, 20, dtype=torch.int32),
                              0, tmp_path)
    q = rs.standard_normal(16).astype(np.float32)
    s = arc.score_boundary_tokens(1, q, [3, 7])
    assert np.allclose(s, k[0, 1, [3, 7]].astype(np.float32) @ q, rtol=1e-6)
    assert arc.score_boundary_tokens(0, q, []).size == 0


@pytest.mark.gpu
def test_compress_async_equals_sync():
    w = numpy_workload(17, 1, 2, 8, 900, 128, 0)
    cfg = TierConfig()
    ref, asy = FoveatedKVCache(cfg), FoveatedKVCache(cfg)
    side = torch.cuda.Stream()
    for i in range(3):
        k = torch.from_numpy(w["k"]).cuda() * (i + 1)
        v = torch.from_numpy(w["v"]).cuda() - i
        ref.update(k, v, i)
        asy.update(k.clone(), v.clone(), i)
        asy.compress_async(i, side)          # overlaps the next "layer's" work
    s1, s2 = ref.compress(), asy.compress()
    torch.cuda.synchronize()
    assert s1["compressed"] and s2["compressed"]
    assert abs(s1["compression"] - s2["compression"]) < 1e-9
    for a, b in zip(ref.layers, asy.layers):
        for f in ("near_k", "far_k", "far_v", "far_v_scale", "far_v_zero", "far_idx", "archive_k"):
            assert torch.equal(getattr(a, f), getattr(b, f)), f
