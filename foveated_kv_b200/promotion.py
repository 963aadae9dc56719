"""Spike drain + promotion pipeline (mirror of the reference's nanobind class
PromotionPipeline, csrc/bindings.cpp:42-100), backed by libfkv.so's
fkv_promo_* entry points (a C++ worker thread with its own CUDA stream)."""

from __future__ import annotations

import ctypes as C
from typing import Optional

import numpy as np
import torch

from . import _native

STAT_KEYS = ("spikes_detected", "spikes_queued", "spikes_deduplicated", "spikes_cooled_down",
             "promotions_completed", "promotions_headroom_full")


def _host_i32(x) -> np.ndarray:
    if isinstance(x, torch.Tensor):
        x = x.detach().to("cpu")
        return np.ascontiguousarray(x.numpy().astype(np.int32, copy=False))
    return np.ascontiguousarray(np.asarray(x, dtype=np.int32))


class PromotionPipeline:
    """Filters per-head spike flags and promotes exact fp16 rows of the
    archive into near-tier headroom, bumping near_valid[b, h] after each row.

    Contract (docs/async_tier_manager.md of the reference): the fused kernel
    reads near_valid once per launch; the pipeline is its only writer after
    register_blob and only appends.  Call ``flush(stream)`` to make a stream
    wait for every queued promotion (deterministic mode); without it a decode
    launch sees each promotion one or more steps later.
    """

    def __init__(self, n_layers: int, cooldown_steps: int = 5, max_per_drain: int = 8,
                 device: Optional[int] = None):
        lib = _native.load()
        dev = torch.cuda.current_device() if device is None and torch.cuda.is_available() else (
            device if device is not None else 0)
        self._h = lib.fkv_promo_create(n_layers, cooldown_steps, max_per_drain, int(dev))
        if not self._h:
            raise _native.FkvNativeError(lib.fkv_last_error().decode())
        self.n_layers = n_layers
        self._keep = {}        # host buffers the C++ side points into
        self._far_idx = {}     # cached host copies of far_idx per layer

    # ---- registration -----------------------------------------------------------
    def register_archive(self, layer_idx: int, path_k: str, path_v: str, H_kv: int, S_arc: int,
                         D: int, archive_idx, B: int = 1):
        """Disk archive: files of (B, H_kv, S_arc, D) fp16 (B=1 is the reference's
        (H_kv, S_arc, D) layout, disk_archive.py:127-185)."""
        idx = _host_i32(archive_idx).reshape(-1)
        self._keep[("idx", layer_idx)] = idx
        _native.check(_native.load().fkv_promo_register_archive(
            self._h, layer_idx, path_k.encode(), path_v.encode(), B, H_kv, S_arc, D,
            idx.ctypes.data, idx.size), "fkv_promo_register_archive")

    def register_archive_host(self, layer_idx: int, archive_k, archive_v, archive_idx):
        """Host-memory archive (B, H_kv, S_arc, D) fp16 (torch CPU tensor,
        ideally pinned, or numpy); the pipeline keeps a reference."""
        k = archive_k.detach().cpu().contiguous() if isinstance(archive_k, torch.Tensor) else \
            torch.from_numpy(np.ascontiguousarray(archive_k))
        v = archive_v.detach().cpu().contiguous() if isinstance(archive_v, torch.Tensor) else \
            torch.from_numpy(np.ascontiguousarray(archive_v))
        B, H, S, D = k.shape
        idx = _host_i32(archive_idx).reshape(-1)
        self._keep[("arc", layer_idx)] = (k, v, idx)
        _native.check(_native.load().fkv_promo_register_archive_host(
            self._h, layer_idx, k.data_ptr() if k.numel() else None,
            v.data_ptr() if v.numel() else None, B, H, S, D, idx.ctypes.data, idx.size),
            "fkv_promo_register_archive_host")

    def register_blob(self, layer_idx: int, info: dict):
        """``info`` = FoveatedLayer.get_blob_info()."""
        _native.check(_native.load().fkv_promo_register_blob(
            self._h, layer_idx, info["near_k"].data_ptr(), info["near_v"].data_ptr(),
            info["near_valid"].data_ptr(), info["B"], info["H_kv"], info["N_near_alloc"],
            info["D"]), "fkv_promo_register_blob")
        self._keep[("blob", layer_idx)] = info

    # ---- per step -------------------------------------------------------------------
    def drain_spikes(self, layer_idx: int, spike_flags, spike_tokens, far_idx,
                     current_step: int) -> int:
        """Filter one layer's spike outputs (B, Hq) and queue promotions;
        returns the number queued.  ``far_idx`` (B, H_kv, F) is copied to the
        host once per layer and cached."""
        fl = _host_i32(spike_flags)
        tk = _host_i32(spike_tokens)
        B, Hq = fl.shape
        key = (layer_idx, id(far_idx))
        fi = self._far_idx.get(key)
        if fi is None:
            fi = _host_i32(far_idx)
            self._far_idx = {k: v for k, v in self._far_idx.items() if k[0] != layer_idx}
            self._far_idx[key] = fi
        H_kv, F = fi.shape[1], fi.shape[2]
        return _native.check(_native.load().fkv_promo_drain(
            self._h, layer_idx, fl.ctypes.data, tk.ctypes.data, fi.ctypes.data if fi.size else None,
            B, Hq, H_kv, F, int(current_step)), "fkv_promo_drain")

    def flush(self, stream: Optional[torch.cuda.Stream] = None, timeout_ms: int = 10000):
        """Wait (bounded) until queued promotions are issued, then make
        ``stream`` (default: current stream) wait for them on the device."""
        st = (stream or torch.cuda.current_stream()).cuda_stream if torch.cuda.is_available() \
            else None
        _native.check(_native.load().fkv_promo_flush(self._h, st, int(timeout_ms)),
                      "fkv_promo_flush")

    def get_stats(self) -> dict:
        arr = (C.c_uint64 * 6)()
        _native.check(_native.load().fkv_promo_stats(self._h, arr), "fkv_promo_stats")
        return dict(zip(STAT_KEYS, (int(x) for x in arr)))

    def stop(self):
        if self._h:
            _native.check(_native.load().fkv_promo_stop(self._h), "fkv_promo_stop")

    def close(self):
        if self._h:
            _native.load().fkv_promo_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
