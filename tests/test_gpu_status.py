"""Kernel status reporting and the strided record merge.

* Every progress wait inside the fused decode kernel is bounded; when one
  runs out the kernel records FKV_ERR_TIMEOUT in the workspace status word,
  lets its copies in flight land and exits.  The test makes a wait run out
  without any fault: FKV_TEST_STALL has the consumers first wait on a barrier
  that nothing completes, with a small wait limit.  The status read through
  the C ABI must then be FKV_ERR_TIMEOUT, and the next normal call on the same
  workspace must succeed with status 0 and correct outputs.
* fkv_combine_partials_strided reads each shard's records in place; record
  blocks at rank strides that are not multiples of 4 floats are only 4-byte
  aligned, and the merge must equal the dense fkv_combine_partials.
"""

import ctypes as C

import numpy as np
import pytest
import torch

from oracle import fkv_oracle as O
from foveated_kv_b200 import TierConfig, compress_layer, _native
from foveated_kv_b200.synthetic import numpy_workload
from tests.helpers import np_, layer_to_oracle, assert_output_close, assert_spikes_match

pytestmark = pytest.mark.gpu


def _decode_raw(lib, lay, q, ws, wait_limit=0, test_flags=0, splits=0):
    B, Hq, D = q.shape
    sh = lay._fill_shape(Hq, 0.5)
    sh.wait_limit, sh.test_flags, sh.num_splits = wait_limit, test_flags, splits
    out = torch.empty((B, Hq, D), dtype=torch.float16, device="cuda")
    fl = torch.empty((B, Hq), dtype=torch.int32, device="cuda")
    tk = torch.empty_like(fl)
    p = lambda x: x.data_ptr()
    dk = p(lay._dec_k) if lay.n_decode else None
    dv = p(lay._dec_v) if lay.n_decode else None
    rc = lib.fkv_decode_fp8(C.byref(sh), p(lay.near_k), p(lay.near_v), p(lay.near_valid),
                            p(lay.far_k), p(lay.far_v), p(lay.far_v_scale), p(lay.far_v_zero),
                            p(q), dk, dv, p(out), p(fl), p(tk), p(ws), ws.numel(),
                            torch.cuda.current_stream().cuda_stream)
    _native.check(rc, "fkv_decode_fp8")
    return out, fl, tk


def _status(lib, ws, clear=0):
    st = C.c_int32(123)
    _native.check(lib.fkv_decode_status(ws.data_ptr(), C.byref(st), clear,
                                        torch.cuda.current_stream().cuda_stream),
                  "fkv_decode_status")
    return st.value


@pytest.mark.parametrize("path", ["mma", "tcgen05"])
@pytest.mark.parametrize("splits_hint", ["auto", "one"])
def test_wait_timeout_is_reported_then_next_call_succeeds(path, splits_hint, monkeypatch):
    monkeypatch.setenv("FKV_QK_PATH", path)
    lib = _native.load()
    w = numpy_workload(81, 1, 2, 8, 3000, 128, 4)
    t = {k: torch.from_numpy(v).cuda() for k, v in w.items()}
    lay = compress_layer(t["k"], t["v"], TierConfig(spike_margin=0.5))
    for i in range(4):
        lay.add_token(t["dec_k"][:, :, i:i + 1], t["dec_v"][:, :, i:i + 1])
    sh = lay._fill_shape(8, 0.5)
    ws = torch.zeros(lib.fkv_decode_workspace_bytes(C.byref(sh)), dtype=torch.uint8, device="cuda")
    splits = 1 if splits_hint == "one" else 0
    assert _status(lib, ws) == 0
    _decode_raw(lib, lay, t["q"], ws, wait_limit=1000, test_flags=_native.FKV_TEST_STALL,
                splits=splits)
    torch.cuda.synchronize()
    assert _status(lib, ws) == _native.FKV_ERR_TIMEOUT          # sticky until cleared
    assert _status(lib, ws, clear=1) == _native.FKV_ERR_TIMEOUT
    assert _status(lib, ws) == 0
    # the context is intact and the workspace (split counters) reusable
    out, fl, tk = _decode_raw(lib, lay, t["q"], ws, splits=splits)
    torch.cuda.synchronize()
    assert _status(lib, ws) == 0
    rout, rfl, rtk, diag = O.decode_attend(layer_to_oracle(lay), w["q"], w["dec_k"], w["dec_v"], 0.5)
    assert_output_close(np_(out).astype(np.float64), rout, f"after timeout ({path})")
    assert assert_spikes_match(np_(fl), np_(tk), rfl, rtk, diag, 0.5) == 0


def test_layer_check_decode_raises_on_timeout():
    """The Python surface surfaces the status word: FoveatedLayer.check_decode."""
    w = numpy_workload(82, 1, 2, 8, 1200, 128, 0)
    t = {k: torch.from_numpy(v).cuda() for k, v in w.items()}
    lay = compress_layer(t["k"], t["v"], TierConfig(spike_margin=0.5))
    lay.attend_fused_with_spikes(t["q"])
    lay.check_decode()                     # ok
    orig = lay._fill_shape

    def stalled(Hq, margin):
        s = orig(Hq, margin)
        s.wait_limit, s.test_flags = 1000, _native.FKV_TEST_STALL
        return s
    lay._fill_shape = stalled
    lay.attend_fused_with_spikes(t["q"])
    with pytest.raises(_native.FkvNativeError, match="timeout"):
        lay.check_decode()
    lay._fill_shape = orig
    out, fl, tk = lay.attend_fused_with_spikes(t["q"])
    lay.check_decode()                     # cleared by the raise, ok again
    rout, rfl, rtk, diag = O.decode_attend(layer_to_oracle(lay), w["q"], None, None, 0.5)
    assert_output_close(np_(out).astype(np.float64)[:, :, 0], rout, "after check")


def test_status_rejects_bad_arguments():
    lib = _native.load()
    st = C.c_int32(0)
    assert lib.fkv_decode_status(None, C.byref(st), 0, None) == -1
    ws = torch.zeros(64, dtype=torch.uint8, device="cuda")
    assert lib.fkv_decode_status(ws.data_ptr() + 4, C.byref(st), 0, None) == -1


@pytest.mark.parametrize("extra", [1, 3, 5])
def test_strided_combine_odd_rank_strides(extra):
    """Shard blocks at rank strides of N*(D+4)+extra floats (4-byte aligned
    only) merge exactly like the dense layout."""
    lib = _native.load()
    P, N, D = 3, 40, 128
    g = torch.Generator(device="cuda").manual_seed(5)
    recs = torch.randn((P, N, D + 4), generator=g, device="cuda")
    recs[:, :, 1] = recs[:, :, 1].abs() + 0.5                  # l > 0
    recs[1, 7, 0] = float("-inf")                               # an empty shard record
    args = torch.randint(-1, 1000, (P, N), generator=g, device="cuda", dtype=torch.int32)
    prs, ars = N * (D + 4) + extra, N + extra
    flat = torch.zeros(P * prs, device="cuda")
    aflat = torch.zeros(P * ars, device="cuda", dtype=torch.int32)
    for k in range(P):
        flat[k * prs:k * prs + N * (D + 4)] = recs[k].reshape(-1)
        aflat[k * ars:k * ars + N] = args[k]
    outs = []
    for strided in (False, True):
        out = torch.empty((N, D), dtype=torch.float16, device="cuda")
        fl = torch.empty((N,), dtype=torch.int32, device="cuda")
        tk = torch.empty_like(fl)
        st = torch.cuda.current_stream().cuda_stream
        if strided:
            rc = lib.fkv_combine_partials_strided(P, N, D, flat.data_ptr(), prs, aflat.data_ptr(),
                                                  ars, 0.5, out.data_ptr(), fl.data_ptr(),
                                                  tk.data_ptr(), st)
        else:
            rc = lib.fkv_combine_partials(P, N, D, recs.data_ptr(), args.data_ptr(), 0.5,
                                          out.data_ptr(), fl.data_ptr(), tk.data_ptr(), st)
        _native.check(rc, "combine")
        outs.append((out, fl, tk))
    torch.cuda.synchronize()
    for a, b in zip(*outs):
        assert torch.equal(a, b)
