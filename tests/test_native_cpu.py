"""libfkv.so loads and exports the C ABI of include/fkv.h; host-only entry
points and argument validation run without a GPU."""

import ctypes as C
import json
import os
import re

import pytest

from foveated_kv_b200 import _native, TierConfig

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_symbols():
    with open(os.path.join(ROOT, "include", "fkv.h")) as f:
        src = f.read()
    return sorted(set(re.findall(r"\b(fkv_[a-z0-9_]+)\s*\(", src)))


def test_library_exports_every_declared_symbol():
    lib = C.CDLL(_native.LIB_PATH)
    syms = header_symbols()
    assert len(syms) >= 20
    for s in syms:
        assert hasattr(lib, s), s
    assert set(syms) == set(_native.SIGNATURES), "ctypes table and header disagree"


def test_abi_version_and_error_string():
    lib = _native.load()
    assert lib.fkv_abi_version() == 2
    assert isinstance(lib.fkv_last_error(), bytes)


def test_tier_boundaries_native_matches_reference_grid():
    with open(os.path.join(ROOT, "tests", "golden", "tier_boundaries.json")) as f:
        tbs = json.load(f)
    for e in tbs:
        assert TierConfig(**e["cfg"]).tier_boundaries(e["S"]) == e["tb"], e


def test_config_validation_mirrors_reference():
    with pytest.raises(ValueError):
        TierConfig(compress_method="int8")
    with pytest.raises(ValueError):
        TierConfig(select="random")
    with pytest.raises(ValueError):
        TierConfig(v_group=16)


def test_invalid_arguments_fail_loudly_without_gpu():
    lib = _native.load()
    sh = _native.DecodeShape(B=1, Hq=6, Hk=4, D=128)       # Hq not a multiple of Hk
    rc = lib.fkv_decode_fp8(C.byref(sh), *([None] * 14), 0, None)
    assert rc == -1
    assert b"multiple" in lib.fkv_last_error()
    sh = _native.DecodeShape(B=1, Hq=4, Hk=4, D=96)
    assert lib.fkv_decode_fp8(C.byref(sh), *([None] * 14), 0, None) == -2
    with pytest.raises(_native.FkvNativeError):
        _native.check(-2, "probe")
    L = _native.TierLayout()
    assert lib.fkv_tier_boundaries(-1, 0.1, 4, 32, 0.5, 8, C.byref(L)) == -1


def test_missing_library_raises(tmp_path, monkeypatch):
    monkeypatch.setattr(_native, "_lib", None)
    with pytest.raises(_native.FkvNativeError):
        _native.load(str(tmp_path / "nope.so"))


def test_shape_limits_rejected_before_any_cuda_call():
    lib = _native.load()
    sh = _native.DecodeShape(B=70000, Hq=8, Hk=1, D=128)      # B*Hk beyond the grid limit
    assert lib.fkv_decode_fp8(C.byref(sh), *([None] * 14), 0, None) == -2
    sh = _native.DecodeShape(B=1, Hq=8, Hk=2, D=128, n_near_alloc=10, n_far=5, n_dec=4, dec_stride=2)
    assert lib.fkv_decode_fp8(C.byref(sh), *([None] * 14), 0, None) == -1   # n_dec > capacity
    assert lib.fkv_decode_workspace_bytes(C.byref(sh)) == 0
    L = _native.TierLayout()
    assert lib.fkv_compress_fp8(C.byref(L), 1, 1, 96, None, None, 0, None, None, 0,
                                *([None] * 8), None) == -2          # head dim 96 unsupported


def test_strided_combine_and_path_query_validate_without_gpu():
    lib = _native.load()
    dummy = C.c_void_p(16)          # never dereferenced: validation fails first
    # rank strides smaller than one shard's records are rejected
    rc = lib.fkv_combine_partials_strided(2, 4, 128, dummy, 4 * 132 - 1, dummy, 4, 0.5,
                                          dummy, dummy, dummy, None)
    assert rc == -1 and b"stride" in lib.fkv_last_error()
    assert lib.fkv_combine_partials_strided(2, 4, 96, dummy, 10**6, dummy, 10**6, 0.5,
                                            dummy, dummy, dummy, None) == -2
    assert lib.fkv_combine_partials_strided(0, 4, 128, dummy, 10**6, dummy, 10**6, 0.5,
                                            dummy, dummy, dummy, None) == -1
    # the q.K path query validates the shape first
    sh = _native.DecodeShape(B=1, Hq=6, Hk=4, D=128)
    assert lib.fkv_decode_qk_path(C.byref(sh), None) == -1
    sh = _native.DecodeShape(B=1, Hq=8, Hk=2, D=64, n_far=100)
    assert lib.fkv_decode_qk_path(C.byref(sh), None) == 0      # D = 64: mma.sync path only
