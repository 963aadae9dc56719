"""GPU edge cases: empty and over-full near tiers, turbo with two q-head
groups and no far tier, strided prefill buffers, and the kernel status word."""

import ctypes as C

import numpy as np
import pytest
import torch

from oracle import fkv_oracle as O
from foveated_kv_b200 import TierConfig, compress_layer, _native
from foveated_kv_b200.cache import _Workspace
from foveated_kv_b200.turbo_constants import host_constants
from foveated_kv_b200.synthetic import numpy_workload
from tests.helpers import np_, bits, layer_to_oracle, assert_output_close, assert_spikes_match

pytestmark = pytest.mark.gpu


def _t(w):
    return {k: torch.from_numpy(v).cuda() for k, v in w.items()}


def test_near_valid_zero_and_clamped():
    w = numpy_workload(81, 2, 2, 8, 500, 128, 3)
    t = _t(w)
    lay = compress_layer(t["k"], t["v"], TierConfig(spike_margin=0.5))
    for i in range(3):
        lay.add_token(t["dec_k"][:, :, i:i + 1], t["dec_v"][:, :, i:i + 1])
    lay.near_valid[0, 0] = 0                       # no near rows for this stream
    lay.near_valid[1, 1] = lay.n_near_alloc + 100  # beyond the allocation: clamped to Np
    out, fl, tk = lay.attend_fused_with_spikes(t["q"])
    torch.cuda.synchronize()
    ref = layer_to_oracle(lay)
    ref["near_valid"] = np.minimum(ref["near_valid"], lay.n_near_alloc)
    rout, rfl, rtk, diag = O.decode_attend(ref, w["q"], w["dec_k"], w["dec_v"], 0.5)
    assert_output_close(np_(out).astype(np.float64)[:, :, 0], rout, "near_valid edges")
    assert assert_spikes_match(np_(fl), np_(tk), rfl, rtk, diag, 0.5) == 0


@pytest.mark.parametrize("S,kw", [(3000, dict()), (40, dict(near_pct=0.9))])
def test_turbo_two_head_groups_and_no_far(S, kw):
    w = numpy_workload(83, 1, 1, 16, S, 64, 2)
    t = _t(w)
    lay = compress_layer(t["k"], t["v"], TierConfig(compress_method="turbo", spike_margin=0.5, **kw))
    for i in range(2):
        lay.add_token(t["dec_k"][:, :, i:i + 1], t["dec_v"][:, :, i:i + 1])
    out, fl, tk = lay.attend_fused_with_spikes(t["q"])
    torch.cuda.synchronize()
    pi, s, c, b = host_constants(64)
    tc = {"Pi": pi, "S": s, "centroids": c, "boundaries": b}
    rout, rfl, rtk, diag = O.decode_attend(layer_to_oracle(lay, tc), w["q"], w["dec_k"], w["dec_v"], 0.5)
    assert_output_close(np_(out).astype(np.float64)[:, :, 0], rout, "turbo G=16")
    assert assert_spikes_match(np_(fl), np_(tk), rfl, rtk, diag, 0.5) == 0


def test_compress_strided_prefill_buffer():
    """K/V rows live in a larger capacity buffer (kv_stride_bh > S*D)."""
    B, H, S, D, cap = 2, 2, 700, 128, 1024
    w = numpy_workload(85, B, H, 8, S, D, 0)
    kbuf = torch.zeros((B, H, cap, D), dtype=torch.float16, device="cuda")
    vbuf = torch.zeros_like(kbuf)
    kbuf[:, :, :S] = torch.from_numpy(w["k"]).cuda()
    vbuf[:, :, :S] = torch.from_numpy(w["v"]).cuda()
    cfg = TierConfig()
    L = cfg.layout(S)
    lib = _native.load()
    Np, F = L.n_near_padded, L.far_count
    ni = torch.empty((B, H, Np), dtype=torch.int32, device="cuda")
    fi = torch.empty((B, H, F), dtype=torch.int32, device="cuda")
    nv = torch.empty((B, H), dtype=torch.int32, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    _native.check(lib.fkv_select_recency(C.byref(L), B, H, ni.data_ptr(), fi.data_ptr(), nv.data_ptr(), st), "sel")
    nk = torch.empty((B, H, Np, D), dtype=torch.float16, device="cuda")
    nvv = torch.empty_like(nk)
    fk = torch.empty((B, H, F, D), dtype=torch.uint8, device="cuda")
    fv = torch.empty((B, H, F, D // 2), dtype=torch.uint8, device="cuda")
    sc = torch.empty((B, H, F), dtype=torch.float16, device="cuda")
    ze = torch.empty_like(sc)
    p = lambda x: x.data_ptr()
    _native.check(lib.fkv_compress_fp8(C.byref(L), B, H, D, p(kbuf), p(vbuf), cap * D, p(ni), p(fi), 0,
                                       p(nk), p(nvv), p(fk), p(fv), p(sc), p(ze), None, None, st), "cmp")
    torch.cuda.synchronize()
    ref = O.compress_layer(w["k"], w["v"], dict())
    for a, b in [(nk, "near_k"), (fk, "far_k"), (fv, "far_v"), (sc, "far_v_scale"), (ze, "far_v_zero")]:
        assert np.array_equal(bits(np_(a)), bits(ref[b])), b


def test_status_word_stays_zero():
    w = numpy_workload(87, 1, 2, 8, 2000, 128, 0)
    t = _t(w)
    lay = compress_layer(t["k"], t["v"], TierConfig())
    for _ in range(3):
        lay.attend_fused_with_spikes(t["q"])
    torch.cuda.synchronize()
    ws = _Workspace._pool[(torch.cuda.current_device(), torch.cuda.current_stream().cuda_stream)][0]
    assert int(ws[:4].view(torch.int32).item()) == 0
