"""fkv_decode_fp8_noalloc: the allocation-free decode entry point.

It exists for callers that cannot allocate device memory on their decode
path (a serving runtime's pre-planned pool, a plugin host that only lends its
own tensors), so it keeps its split scratch in a fixed array inside
libfkv.so.  Checked here through the C ABI against fkv_decode_fp8 with a
caller workspace, on two calls in a row (the second sees the scratch the
first left behind).  This file is collected last on purpose.
"""

import ctypes as C

import numpy as np
import pytest
import torch

from foveated_kv_b200 import TierConfig, compress_layer, _native
from foveated_kv_b200.synthetic import numpy_workload
from tests.helpers import OUT_MAX_ABS

pytestmark = pytest.mark.gpu


def _layer(seed, B, Hk, Hq, S, D, n_dec):
    w = numpy_workload(seed, B, Hk, Hq, S, D, n_dec)
    t = {k: torch.from_numpy(v).cuda() for k, v in w.items()}
    lay = compress_layer(t["k"], t["v"], TierConfig(spike_margin=0.5))
    for i in range(n_dec):
        lay.add_token(t["dec_k"][:, :, i:i + 1], t["dec_v"][:, :, i:i + 1])
    return lay, t["q"]


def _run(lay, q, noalloc):
    lib = _native.load()
    B, Hq, D = q.shape
    sh = _native.DecodeShape(B=B, Hq=Hq, Hk=lay.H_kv, D=D, n_near_alloc=lay.n_near_alloc,
                             n_far=lay.n_far, n_dec=lay.n_decode, dec_stride=lay._dec_k.shape[2],
                             v_group=0, num_splits=0, spike_margin=0.5)
    out = torch.empty((B, Hq, D), dtype=torch.float16, device="cuda")
    fl = torch.empty((B, Hq), dtype=torch.int32, device="cuda")
    tk = torch.empty_like(fl)
    p = lambda x: x.data_ptr()
    st = torch.cuda.current_stream().cuda_stream
    common = [p(lay.near_k), p(lay.near_v), p(lay.near_valid), p(lay.far_k), p(lay.far_v),
              p(lay.far_v_scale), p(lay.far_v_zero), p(q), p(lay._dec_k), p(lay._dec_v),
              p(out), p(fl), p(tk)]
    if noalloc:
        rc = lib.fkv_decode_fp8_noalloc(C.byref(sh), *common, st)
        _native.check(rc, "fkv_decode_fp8_noalloc")
    else:
        ws = torch.zeros(lib.fkv_decode_workspace_bytes(C.byref(sh)), dtype=torch.uint8,
                         device="cuda")
        rc = lib.fkv_decode_fp8(C.byref(sh), *common, p(ws), ws.numel(), st)
        _native.check(rc, "fkv_decode_fp8")
    torch.cuda.synchronize()
    return out.float().cpu().numpy(), fl.cpu().numpy(), tk.cpu().numpy()


@pytest.mark.parametrize("shape", [(2, 4, 16, 3000, 128, 5), (1, 2, 14, 1024, 64, 16)])
def test_noalloc_matches_workspace_entry_twice(shape):
    lay, q = _layer(31, *shape)
    ref = _run(lay, q, noalloc=False)
    lib = _native.load()
    for _ in range(2):   # second call reuses the scratch left by the first
        got = _run(lay, q, noalloc=True)
        assert np.abs(got[0] - ref[0]).max() <= OUT_MAX_ABS
        assert np.array_equal(got[1], ref[1])
        assert np.array_equal(got[2], ref[2])
        # the kernel status word of the call (kept in the fixed scratch) is clean
        st = C.c_int32(123)
        _native.check(lib.fkv_decode_noalloc_status(C.byref(st),
                                                    torch.cuda.current_stream().cuda_stream),
                      "fkv_decode_noalloc_status")
        assert st.value == 0


def test_noalloc_rejects_oversized_shape():
    lib = _native.load()
    sh = _native.DecodeShape(B=4096, Hq=32, Hk=8, D=128, n_near_alloc=5000, n_far=200000,
                             n_dec=0, dec_stride=0, v_group=0, num_splits=16, spike_margin=0.5)
    rc = lib.fkv_decode_fp8_noalloc(C.byref(sh), *([None] * 13), None)
    assert rc == -1
    assert b"limit" in lib.fkv_last_error()
