"""ctypes binding of libfkv.so (the C ABI in include/fkv.h).

The library is built in-tree (``python -m foveated_kv_b200.build`` or
``__graft_entry__.build()``).  There is no fallback: if the library is missing
or fails to load, every entry point raises ``FkvNativeError``.
"""

from __future__ import annotations

import ctypes as C
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "_lib", "libfkv.so")

FKV_ERRORS = {-1: "invalid argument", -2: "unsupported", -3: "CUDA error", -4: "timeout",
              -5: "I/O error"}


class FkvNativeError(RuntimeError):
    pass


class TierLayout(C.Structure):
    _fields_ = [(n, C.c_int32) for n in (
        "S", "n_sinks", "window", "near_from_mid", "far_count", "r_actual", "n_near_padded",
        "mid_start", "mid_end", "near_mid_start")]

    def as_dict(self) -> dict:
        """Same keys as MLXTierConfig.tier_boundaries (mlx_foveated.py:157-169)."""
        return {"n_sinks": self.n_sinks, "window": self.window,
                "near_from_mid": self.near_from_mid, "far_count": self.far_count,
                "R_actual": self.r_actual, "N_near_padded": self.n_near_padded,
                "mid_start": self.mid_start, "mid_end": self.mid_end,
                "near_mid_start": self.near_mid_start, "far_src_offset": self.mid_start}


class DecodeShape(C.Structure):
    _fields_ = [("B", C.c_int32), ("Hq", C.c_int32), ("Hk", C.c_int32), ("D", C.c_int32),
                ("n_near_alloc", C.c_int32), ("n_far", C.c_int32), ("n_dec", C.c_int32),
                ("dec_stride", C.c_int32), ("v_group", C.c_int32), ("num_splits", C.c_int32),
                ("spike_margin", C.c_float), ("qjl_coef", C.c_float), ("wait_limit", C.c_int32),
                ("test_flags", C.c_int32)]


FKV_TEST_STALL = 1
FKV_ERR_TIMEOUT = -4


P = C.c_void_p
I32 = C.c_int32
I64 = C.c_int64
SZ = C.c_size_t

# name -> (restype, argtypes); every symbol declared in include/fkv.h
SIGNATURES = {
    "fkv_abi_version": (C.c_int, []),
    "fkv_last_error": (C.c_char_p, []),
    "fkv_tier_boundaries": (C.c_int, [I32, C.c_double, I32, I32, C.c_double, I32,
                                      C.POINTER(TierLayout)]),
    "fkv_select_recency": (C.c_int, [C.POINTER(TierLayout), I32, I32, P, P, P, P]),
    "fkv_select_importance_workspace_bytes": (SZ, [C.POINTER(TierLayout), I32, I32, I32]),
    "fkv_select_importance": (C.c_int, [C.POINTER(TierLayout), I32, I32, I32, I32, P, I64, P,
                                        P, P, P, P, SZ, P]),
    "fkv_compress_fp8": (C.c_int, [C.POINTER(TierLayout), I32, I32, I32, P, P, I64, P, P, I32,
                                   P, P, P, P, P, P, P, P, P]),
    "fkv_compress_turbo": (C.c_int, [C.POINTER(TierLayout), I32, I32, I32, P, P, I64, P, P,
                                     P, P, P, P, P, P, P, P, P, P, P, P, P, P, P]),
    "fkv_decode_workspace_bytes": (SZ, [C.POINTER(DecodeShape)]),
    "fkv_decode_qk_path": (C.c_int, [C.POINTER(DecodeShape), P]),
    "fkv_decode_status": (C.c_int, [P, C.POINTER(I32), I32, P]),
    "fkv_decode_plan": (C.c_int, [C.POINTER(DecodeShape), P, I32, P]),
    "fkv_decode_noalloc_status": (C.c_int, [C.POINTER(I32), P]),
    "fkv_decode_fp8": (C.c_int, [C.POINTER(DecodeShape), P, P, P, P, P, P, P, P, P, P, P, P,
                                 P, P, SZ, P]),
    "fkv_decode_turbo": (C.c_int, [C.POINTER(DecodeShape), P, P, P, P, P, P, P, P, P, P, P,
                                   P, P, P, P, P, P, P, P, SZ, P]),
    "fkv_decode_fp8_noalloc": (C.c_int, [C.POINTER(DecodeShape), P, P, P, P, P, P, P, P, P, P,
                                         P, P, P, P]),
    "fkv_decode_fp8_partial": (C.c_int, [C.POINTER(DecodeShape), P, P, P, P, P, P, P, P, P,
                                         P, I32, P, P, P, SZ, P]),
    "fkv_combine_partials": (C.c_int, [I32, I32, I32, P, P, C.c_float, P, P, P, P]),
    "fkv_combine_partials_strided": (C.c_int, [I32, I32, I32, P, C.c_int64, P, C.c_int64, C.c_float,
                                               P, P, P, P]),
    "fkv_exchange_recv_bytes": (SZ, [I32, I32, I32]),
    "fkv_exchange_block_stride": (I64, [I32, I32]),
    "fkv_exchange_combine": (C.c_int, [I32, I32, I32, I32, P, P, P, P, C.c_float, P, P, P, P]),
    "fkv_ipc_handle_bytes": (C.c_int, []),
    "fkv_ipc_get_handle": (C.c_int, [P, P, C.POINTER(I64)]),
    "fkv_ipc_open": (C.c_int, [P, I64, C.POINTER(P)]),
    "fkv_ipc_close": (C.c_int, [P, I64]),
    "fkv_promo_create": (P, [I32, I32, I32, I32]),
    "fkv_promo_register_archive": (C.c_int, [P, I32, C.c_char_p, C.c_char_p, I32, I32, I32,
                                             I32, P, I64]),
    "fkv_promo_register_archive_host": (C.c_int, [P, I32, P, P, I32, I32, I32, I32, P, I64]),
    "fkv_promo_register_blob": (C.c_int, [P, I32, P, P, P, I32, I32, I32, I32]),
    "fkv_promo_drain": (C.c_int, [P, I32, P, P, P, I32, I32, I32, I32, I32]),
    "fkv_promo_flush": (C.c_int, [P, P, I32]),
    "fkv_promo_stats": (C.c_int, [P, P]),
    "fkv_promo_stop": (C.c_int, [P]),
    "fkv_promo_destroy": (None, [P]),
}

_lib = None
_lock = threading.Lock()


def load(path: str = None):
    """Load libfkv.so once; raises FkvNativeError if it is absent or broken.
    FKV_LIBRARY in the environment names another build of the library (for
    A/B timing of builds; entry points it lacks raise when used)."""
    global _lib
    path = path or os.environ.get("FKV_LIBRARY") or LIB_PATH
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(path):
            raise FkvNativeError(
                f"libfkv.so not found at {path}; build it with `python -m foveated_kv_b200.build`")
        try:
            lib = C.CDLL(path)
        except OSError as e:
            raise FkvNativeError(f"failed to load {path}: {e}") from e
        missing = []
        for name, (res, args) in SIGNATURES.items():
            try:
                fn = getattr(lib, name)
            except AttributeError:
                missing.append(name)
                continue
            fn.restype = res
            fn.argtypes = args
        if missing and path == LIB_PATH:
            raise FkvNativeError(f"{path} lacks symbols: {missing}")
        _lib = lib
        return lib


def check(rc: int, what: str):
    if rc < 0:
        msg = load().fkv_last_error().decode(errors="replace")
        raise FkvNativeError(f"{what} failed ({FKV_ERRORS.get(rc, rc)}): {msg}")
    return rc


def tier_layout(S, near_pct, n_sinks, window_size, headroom_pct, headroom_min) -> TierLayout:
    L = TierLayout()
    check(load().fkv_tier_boundaries(int(S), float(near_pct), int(n_sinks), int(window_size),
                                     float(headroom_pct), int(headroom_min), C.byref(L)),
          "fkv_tier_boundaries")
    return L
