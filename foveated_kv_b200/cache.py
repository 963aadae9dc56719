"""Two-tier foveated KV cache on B200 (mirror of MLXFoveatedLayer /
MLXFoveatedKVCache, src/foveated_kv/mlx_foveated.py:172-968).

All tensors are torch CUDA tensors; every computation on them goes through
libfkv.so (include/fkv.h).  There is no host or eager-torch fallback.
"""

from __future__ import annotations

import ctypes as C
import math
from typing import Optional, Sequence

import torch

from . import _native
from .config import TierConfig

F16 = torch.float16
I32 = torch.int32
U8 = torch.uint8


def _p(t: Optional[torch.Tensor]):
    return None if t is None or t.numel() == 0 else t.data_ptr()


def _stream(device=None) -> int:
    return torch.cuda.current_stream(device).cuda_stream


class _Workspace:
    """Zero-initialised scratch shared by the decode calls issued on one
    (device, stream); calls on one stream never overlap, so sharing is safe.

    libfkv keeps split counters at the front and split records at the back of
    the workspace, so one buffer serves every shape as long as it holds the
    largest request seen plus the largest counter region seen (bounded here by
    the largest request)."""

    _pool: dict = {}

    @classmethod
    def get(cls, nbytes: int, device: torch.device) -> torch.Tensor:
        key = (device.index, _stream(device))
        buf, peak = cls._pool.get(key, (None, 0))
        peak = max(peak, nbytes)
        need = 2 * peak
        if buf is None or buf.numel() < need:
            buf = torch.zeros(max(need, 1 << 16), dtype=U8, device=device)
        cls._pool[key] = (buf, peak)
        return buf


def workspace_status(device: torch.device, clear: bool = True) -> int:
    """Kernel status word of the shared decode workspace of (device, current
    stream): 0 = every launch since the last clear completed its waits."""
    key = (device.index, _stream(device))
    buf = _Workspace._pool.get(key, (None, 0))[0]
    if buf is None:
        return 0
    lib = _native.load()
    st = C.c_int32(0)
    _native.check(lib.fkv_decode_status(buf.data_ptr(), C.byref(st), int(clear), key[1]),
                  "fkv_decode_status")
    return int(st.value)


class FoveatedLayer:
    """Single-layer two-tier store (near fp16 + far fp8/INT4 or TurboQuant).

    Shapes (B batch, H KV heads, Np = R + headroom, F far tokens):
      near_k, near_v   (B, H, Np, D) fp16, rows >= near_valid[b, h] are headroom
      near_idx         (B, H, Np) int32 token positions, -1 in headroom
      near_valid       (B, H) int32 (the reference keeps (H,), shared by the batch)
      far_k            (B, H, F, D) uint8 E4M3;  far_v (B, H, F, D/2) uint8
      far_v_scale/zero (B, H, F) fp16, or (B, H, F, D/32) with v_group=32
      far_idx          (B, H, F) int32
      archive_k/v      (B, H, F, D) fp16 exact far rows (promotion source)
      turbo_*          TurboQuant far tier when compress_method == 'turbo'
    """

    def __init__(self, *, near_k, near_v, near_idx, near_valid, far_idx, archive_k=None,
                 archive_v=None, archive_idx=None, compress_method="fp8", far_k=None,
                 far_v=None, far_v_scale=None, far_v_zero=None, v_group=None,
                 turbo_far_k_indices=None, turbo_far_k_signs=None, turbo_far_k_norm=None,
                 turbo_far_k_gamma=None, turbo_far_v_packed=None, turbo_far_v_scale=None,
                 turbo_constants=None, spike_margin: float = 10.0,
                 qjl_coef: float = 1.2533141373155001):
        self.near_k, self.near_v, self.near_idx = near_k, near_v, near_idx
        self.near_valid = near_valid
        self.far_idx = far_idx
        self.archive_k, self.archive_v = archive_k, archive_v
        self.archive_idx = far_idx if archive_idx is None else archive_idx
        self.compress_method = compress_method
        self.far_k, self.far_v = far_k, far_v
        self.far_v_scale, self.far_v_zero = far_v_scale, far_v_zero
        self.v_group = v_group
        self.turbo_far_k_indices = turbo_far_k_indices
        self.turbo_far_k_signs = turbo_far_k_signs
        self.turbo_far_k_norm = turbo_far_k_norm
        self.turbo_far_k_gamma = turbo_far_k_gamma
        self.turbo_far_v_packed = turbo_far_v_packed
        self.turbo_far_v_scale = turbo_far_v_scale
        self._turbo_constants = turbo_constants
        self.spike_margin = float(spike_margin)
        self.qjl_coef = float(qjl_coef)
        B, H, Np, D = near_k.shape
        self.B, self.H_kv, self.D = B, H, D
        self.n_near_alloc = Np
        self.n_far = far_idx.shape[2]
        self.device = near_k.device
        self._dec_k = torch.zeros((B, H, 16, D), dtype=F16, device=self.device)
        self._dec_v = torch.zeros_like(self._dec_k)
        self._n_dec = 0
        self._shape = _native.DecodeShape()
        self._nv_snapshot = None
        self._next_pos = int(max(int(near_idx.max().item()) if near_idx.numel() else -1,
                                 int(far_idx.max().item()) if far_idx.numel() else -1)) + 1

    # ---- decode buffer (mlx_foveated.py:404-428) ------------------------------
    def add_token(self, new_k: torch.Tensor, new_v: torch.Tensor) -> None:
        """Append one decode token (B, H, 1, D) to the fp16 decode buffer."""
        n = new_k.shape[2]
        if self._n_dec + n > self._dec_k.shape[2]:
            cap = max(2 * self._dec_k.shape[2], self._n_dec + n)
            nk = torch.zeros((self.B, self.H_kv, cap, self.D), dtype=F16, device=self.device)
            nv = torch.zeros_like(nk)
            nk[:, :, :self._n_dec] = self._dec_k[:, :, :self._n_dec]
            nv[:, :, :self._n_dec] = self._dec_v[:, :, :self._n_dec]
            self._dec_k, self._dec_v = nk, nv
        self._dec_k[:, :, self._n_dec:self._n_dec + n] = new_k.to(F16)
        self._dec_v[:, :, self._n_dec:self._n_dec + n] = new_v.to(F16)
        self._n_dec += n
        self._next_pos += n

    @property
    def decode_k(self) -> Optional[torch.Tensor]:
        return None if self._n_dec == 0 else self._dec_k[:, :, :self._n_dec]

    @property
    def decode_v(self) -> Optional[torch.Tensor]:
        return None if self._n_dec == 0 else self._dec_v[:, :, :self._n_dec]

    @property
    def n_decode(self) -> int:
        return self._n_dec

    @property
    def total_tokens(self) -> int:
        return int(self.near_valid.max().item()) + self.n_far

    @property
    def effective_near_k(self) -> torch.Tensor:
        mv = int(self.near_valid.max().item())
        nk = self.near_k[:, :, :mv]
        return nk if self._n_dec == 0 else torch.cat([nk, self.decode_k], dim=2)

    @property
    def effective_near_v(self) -> torch.Tensor:
        mv = int(self.near_valid.max().item())
        nv = self.near_v[:, :, :mv]
        return nv if self._n_dec == 0 else torch.cat([nv, self.decode_v], dim=2)

    # ---- fused decode (mlx_foveated.py:372-402) --------------------------------
    def _fill_shape(self, Hq: int, margin: float) -> _native.DecodeShape:
        s = self._shape
        s.B, s.Hq, s.Hk, s.D = self.B, Hq, self.H_kv, self.D
        s.n_near_alloc, s.n_far, s.n_dec = self.n_near_alloc, self.n_far, self._n_dec
        s.dec_stride = self._dec_k.shape[2]
        s.v_group = int(self.v_group or 0)
        s.num_splits = 0
        s.spike_margin = margin
        s.qjl_coef = self.qjl_coef
        s.wait_limit = 0
        s.test_flags = 0
        return s

    def attend_fused_with_spikes(self, query: torch.Tensor, spike_margin: Optional[float] = None,
                                 out: Optional[torch.Tensor] = None):
        """Fused decode attention + spike detection.

        query (B, Hq, 1, D) (or (B, Hq, D)); returns (out (B, Hq, 1, D) fp16,
        spike_flags (B, Hq) int32, spike_tokens (B, Hq) int32 far-local or -1).
        ``spike_margin`` overrides the layer's margin when given (the
        reference ignores this argument and always uses 10.0).
        """
        lib = _native.load()
        if not (query.is_cuda and self.near_k.is_cuda) or query.device != self.near_k.device:
            raise ValueError("attend_fused_with_spikes: query and tiers must be CUDA tensors "
                             "on the same device")
        B, Hq, D = query.shape[0], query.shape[1], query.shape[-1]
        q = query.reshape(B, Hq, D)
        if q.dtype != F16 or not q.is_contiguous():
            q = q.to(F16).contiguous()
        margin = self.spike_margin if spike_margin is None else float(spike_margin)
        sh = self._fill_shape(Hq, margin)
        key = (Hq, self._n_dec, sh.dec_stride)
        if getattr(self, "_ws_key", None) != key:      # plan changes only with these
            self._ws_key = key
            self._ws_bytes = lib.fkv_decode_workspace_bytes(C.byref(sh))
        ws = _Workspace.get(self._ws_bytes, self.device)
        if out is None:
            out = torch.empty((B, Hq, 1, D), dtype=F16, device=self.device)
        flags = torch.empty((B, Hq), dtype=I32, device=self.device)
        tokens = torch.empty((B, Hq), dtype=I32, device=self.device)
        dk = self._dec_k if self._n_dec else None
        dv = self._dec_v if self._n_dec else None
        st = _stream(self.device)
        nv = self.near_valid
        if self._nv_snapshot is not None:
            # a promotion worker may bump near_valid while this launch runs:
            # every CTA of the launch must see one count per stream, so the
            # launch reads a snapshot taken in stream order just before it
            self._nv_snapshot.copy_(self.near_valid)
            nv = self._nv_snapshot
        if self.compress_method == "turbo":
            tc = self._turbo_constants
            rc = lib.fkv_decode_turbo(
                C.byref(sh), _p(self.near_k), _p(self.near_v), _p(nv),
                _p(self.turbo_far_k_indices), _p(self.turbo_far_k_signs),
                _p(self.turbo_far_k_norm), _p(self.turbo_far_k_gamma),
                _p(self.turbo_far_v_packed), _p(self.turbo_far_v_scale), _p(tc.Pi), _p(tc.S),
                _p(tc.centroids), _p(q), _p(dk), _p(dv), _p(out), _p(flags), _p(tokens),
                ws.data_ptr(), ws.numel(), st)
            _native.check(rc, "fkv_decode_turbo")
        else:
            rc = lib.fkv_decode_fp8(
                C.byref(sh), _p(self.near_k), _p(self.near_v), _p(nv),
                _p(self.far_k), _p(self.far_v), _p(self.far_v_scale), _p(self.far_v_zero), _p(q),
                _p(dk), _p(dv), _p(out), _p(flags), _p(tokens), ws.data_ptr(), ws.numel(), st)
            _native.check(rc, "fkv_decode_fp8")
        return out, flags, tokens

    def decode_status(self, clear: bool = True) -> int:
        """Status word of the fused decode calls issued on the current stream
        since it was last cleared: 0, or -4 (FKV_ERR_TIMEOUT) when a bounded
        wait inside a launch expired (that launch's outputs are not valid).
        Waits for the stream."""
        return workspace_status(self.device, clear)

    def check_decode(self) -> None:
        """Raise FkvNativeError if a decode launch on the current stream timed out."""
        st = self.decode_status(clear=True)
        if st != 0:
            raise _native.FkvNativeError(
                f"fused decode kernel reported status {st} ({_native.FKV_ERRORS.get(st, st)})")

    def attend_fused(self, query: torch.Tensor) -> torch.Tensor:
        return self.attend_fused_with_spikes(query)[0]

    def attend(self, query: torch.Tensor) -> torch.Tensor:
        """Attention over near + far + decode buffer (the fused kernel; the
        reference's dequantise-then-SDPA path is not kept in the product)."""
        return self.attend_fused(query)

    # ---- alternative spike policy (mlx_foveated.py:451-499) -----------------------
    def detect_spikes(self, query: torch.Tensor, margin: float = 0.5) -> Optional[torch.Tensor]:
        """GQA-mean query spike check (``detect_spikes``, mlx_foveated.py:451-490).

        q = mean of each group's query heads (rounded to fp16, the query
        dtype); a (b, kv head) spikes when some far score exceeds its lowest
        near / decode score + margin, and reports its far-local argmax
        (earliest on ties).  Runs as ONE fused decode launch with the mean
        queries as one query head per KV head: the kernel's spike emission is
        exactly this test (its attention output is discarded).  Returns an
        int32 (N, 3) tensor of [b, kv head, far-local argmax], or None.
        """
        if self.compress_method != "fp8" or self.n_far == 0:
            return None
        B, D = query.shape[0], query.shape[-1]
        q = query.reshape(B, query.shape[1], D).float()
        G = q.shape[1] // self.H_kv
        qm = q.reshape(B, self.H_kv, G, D).mean(2).to(F16).contiguous()       # (B, H, D)
        _, flags, tokens = self.attend_fused_with_spikes(qm, spike_margin=margin)
        bh = flags.nonzero()
        if bh.numel() == 0:
            return None
        return torch.cat([bh, tokens[bh[:, 0], bh[:, 1]][:, None]], 1).to(torch.int32)

    # ---- promotion target (foveated_attn.cpp:242-254) ---------------------------
    def get_blob_info(self) -> dict:
        """Promotion target (the worker writes near_k / near_v rows and
        near_valid).  From here on the fused decode reads a per-launch
        snapshot of near_valid, so promotions landing during a launch cannot
        give its CTAs different counts (the reference's kernel reads
        near_valid once per dispatch)."""
        if self._nv_snapshot is None:
            self._nv_snapshot = torch.empty_like(self.near_valid)
        return {"near_k": self.near_k, "near_v": self.near_v, "near_valid": self.near_valid,
                "N_near_alloc": self.n_near_alloc, "B": self.B, "H_kv": self.H_kv, "D": self.D}

    def memory_bytes(self) -> dict:
        """Same accounting as MLXFoveatedLayer.memory_bytes (mlx_foveated.py:501-525)."""
        nb = lambda t: 0 if t is None else t.numel() * t.element_size()
        near = nb(self.near_k) + nb(self.near_v)
        if self.compress_method == "turbo":
            far = sum(nb(t) for t in (self.turbo_far_k_indices, self.turbo_far_k_signs,
                                      self.turbo_far_k_norm, self.turbo_far_k_gamma,
                                      self.turbo_far_v_packed, self.turbo_far_v_scale))
        else:
            far = nb(self.far_k) + nb(self.far_v) + nb(self.far_v_scale) + nb(self.far_v_zero)
        arc = nb(self.archive_k) + nb(self.archive_v)
        return {"near": near, "far": far, "archive": arc, "total_quantized": near + far,
                "total_with_archive": near + far + arc}


def compress_layer(keys: torch.Tensor, values: torch.Tensor, cfg: TierConfig,
                   query: Optional[torch.Tensor] = None, keep_archive: bool = True,
                   stream: Optional[int] = None) -> FoveatedLayer:
    """Tier one layer's prefill K/V (B, H, S, D) on the device.

    Mirrors _assign_and_build_layer (mlx_foveated.py:799-944) / the C++
    CompressHandle (foveated_compress.cpp:95-201): selection, gather, encode
    and archive copy run as two launches (select, then one fused pass).
    """
    lib = _native.load()
    if not keys.is_cuda:
        raise ValueError("keys/values must be CUDA tensors")
    k = keys.to(F16).contiguous()
    v = values.to(F16).contiguous()
    B, H, S, D = k.shape
    dev = k.device
    L = cfg.layout(S)
    Np, F = L.n_near_padded, L.far_count
    st = _stream(dev) if stream is None else stream
    near_idx = torch.empty((B, H, Np), dtype=I32, device=dev)
    far_idx = torch.empty((B, H, F), dtype=I32, device=dev)
    near_valid = torch.empty((B, H), dtype=I32, device=dev)
    if cfg.select == "importance":
        if query is None:
            raise ValueError("select='importance' needs the observation query (B, Hq, D)")
        q = query.reshape(B, query.shape[1], D).to(F16).contiguous()
        ws_b = lib.fkv_select_importance_workspace_bytes(C.byref(L), B, H, q.shape[1])
        ws = torch.zeros(max(ws_b, 16), dtype=U8, device=dev)
        _native.check(lib.fkv_select_importance(
            C.byref(L), B, H, q.shape[1], D, _p(k), S * D, _p(q), _p(near_idx), _p(far_idx),
            _p(near_valid), ws.data_ptr(), ws.numel(), st), "fkv_select_importance")
    else:
        _native.check(lib.fkv_select_recency(C.byref(L), B, H, _p(near_idx), _p(far_idx),
                                             _p(near_valid), st), "fkv_select_recency")
    near_k = torch.empty((B, H, Np, D), dtype=F16, device=dev)
    near_v = torch.empty_like(near_k)
    arc_k = torch.empty((B, H, F, D), dtype=F16, device=dev) if keep_archive else None
    arc_v = torch.empty_like(arc_k) if keep_archive else None
    common = dict(near_k=near_k, near_v=near_v, near_idx=near_idx, near_valid=near_valid,
                  far_idx=far_idx, archive_k=arc_k, archive_v=arc_v,
                  spike_margin=cfg.spike_margin, qjl_coef=cfg.qjl_coef)
    if cfg.compress_method == "turbo":
        from .turbo_constants import get_turbo_constants
        tc = get_turbo_constants(D, str(dev))
        ki = torch.empty((B, H, F, D // 4), dtype=U8, device=dev)
        ks = torch.empty((B, H, F, D // 8), dtype=U8, device=dev)
        kn = torch.empty((B, H, F), dtype=F16, device=dev)
        kg = torch.empty((B, H, F), dtype=F16, device=dev)
        vp = torch.empty((B, H, F, D // 4), dtype=U8, device=dev)
        vs = torch.empty((B, H, F, D // 32), dtype=F16, device=dev)
        _native.check(lib.fkv_compress_turbo(
            C.byref(L), B, H, D, _p(k), _p(v), S * D, _p(near_idx), _p(far_idx), _p(tc.Pi),
            _p(tc.S), _p(tc.centroids), _p(tc.boundaries), _p(near_k), _p(near_v), _p(ki),
            _p(ks), _p(kn), _p(kg), _p(vp), _p(vs), _p(arc_k), _p(arc_v), st),
            "fkv_compress_turbo")
        return FoveatedLayer(compress_method="turbo", turbo_far_k_indices=ki,
                             turbo_far_k_signs=ks, turbo_far_k_norm=kn, turbo_far_k_gamma=kg,
                             turbo_far_v_packed=vp, turbo_far_v_scale=vs, turbo_constants=tc,
                             far_k=torch.zeros((B, H, 0, D), dtype=U8, device=dev),
                             **common)
    vg = cfg.v_group
    far_k = torch.empty((B, H, F, D), dtype=U8, device=dev)
    far_v = torch.empty((B, H, F, D // 2), dtype=U8, device=dev)
    sshape = (B, H, F) if vg is None else (B, H, F, D // vg)
    vsc = torch.empty(sshape, dtype=F16, device=dev)
    vze = torch.empty(sshape, dtype=F16, device=dev)
    _native.check(lib.fkv_compress_fp8(
        C.byref(L), B, H, D, _p(k), _p(v), S * D, _p(near_idx), _p(far_idx), int(vg or 0),
        _p(near_k), _p(near_v), _p(far_k), _p(far_v), _p(vsc), _p(vze), _p(arc_k), _p(arc_v),
        st), "fkv_compress_fp8")
    return FoveatedLayer(compress_method="fp8", far_k=far_k, far_v=far_v, far_v_scale=vsc,
                         far_v_zero=vze, v_group=vg, **common)


class FoveatedKVCache:
    """Multi-layer cache: ``update`` collects prefill K/V per layer,
    ``compress`` tiers every layer (MLXFoveatedKVCache, mlx_foveated.py:603-968)."""

    def __init__(self, cfg: Optional[TierConfig] = None):
        self.cfg = cfg or TierConfig()
        self.layers: list = []
        self._prefill_keys: list = []
        self._prefill_values: list = []
        self._compressed = False
        self.seq_length = 0

    def update(self, key_states: torch.Tensor, value_states: torch.Tensor, layer_idx: int):
        while len(self._prefill_keys) <= layer_idx:
            self._prefill_keys.append(None)
            self._prefill_values.append(None)
            self.layers.append(None)
        if self._prefill_keys[layer_idx] is None:
            self._prefill_keys[layer_idx] = key_states
            self._prefill_values[layer_idx] = value_states
        else:
            self._prefill_keys[layer_idx] = torch.cat([self._prefill_keys[layer_idx], key_states], 2)
            self._prefill_values[layer_idx] = torch.cat(
                [self._prefill_values[layer_idx], value_states], 2)

    def compress_async(self, layer_idx: int, stream: Optional[torch.cuda.Stream] = None,
                       query=None, keep_archive: bool = True) -> torch.cuda.Event:
        """Tier one layer on a side stream as soon as its prefill K/V is
        complete, so the compression overlaps the next layer's prefill on the
        main stream.  Returns an event recorded after the layer's compression;
        ``compress()`` (or ``synchronize_compression``) waits for all of them."""
        k, v = self._prefill_keys[layer_idx], self._prefill_values[layer_idx]
        main = torch.cuda.current_stream(k.device)
        side = stream or torch.cuda.Stream(k.device)
        side.wait_stream(main)                       # K/V were produced on main
        with torch.cuda.stream(side):
            lay = compress_layer(k, v, self.cfg, query, keep_archive)
        k.record_stream(side)
        v.record_stream(side)
        ev = torch.cuda.Event()
        ev.record(side)
        self.layers[layer_idx] = lay
        self._pending = getattr(self, "_pending", {})
        self._pending[layer_idx] = (ev, k.numel() * k.element_size() * 2, k.shape[2])
        self._prefill_keys[layer_idx] = None
        self._prefill_values[layer_idx] = None
        return ev

    def synchronize_compression(self) -> None:
        """Make the current stream wait for every ``compress_async`` layer."""
        for ev, _, _ in getattr(self, "_pending", {}).values():
            torch.cuda.current_stream().wait_event(ev)

    def compress(self, query=None, keep_archive: bool = True) -> dict:
        """Compress all layers.  ``query``: observation query for importance
        selection -- one (B, Hq, D) tensor for every layer, or a per-layer list."""
        pending = getattr(self, "_pending", {})
        if not self._prefill_keys and not pending:
            return {"compressed": False}
        self.synchronize_compression()
        before = after = 0
        for i, (_, nbytes, S) in pending.items():
            before += nbytes
            after += self.layers[i].memory_bytes()["total_quantized"]
            self.seq_length = S
        self._pending = {}
        for i, (k, v) in enumerate(zip(self._prefill_keys, self._prefill_values)):
            if k is None:
                continue
            q = query[i] if isinstance(query, (list, tuple)) else query
            lay = compress_layer(k, v, self.cfg, q, keep_archive)
            self.layers[i] = lay
            self.seq_length = k.shape[2]
            before += k.numel() * k.element_size() * 2
            after += lay.memory_bytes()["total_quantized"]
        self._prefill_keys.clear()
        self._prefill_values.clear()
        self._compressed = True
        return {"compressed": True, "n_layers": len(self.layers),
                "before_mb": before / (1024 * 1024), "after_mb": after / (1024 * 1024),
                "compression": before / max(after, 1)}

    def attend(self, layer_idx: int, query: torch.Tensor) -> torch.Tensor:
        lay = self.layers[layer_idx]
        if lay is None:
            raise ValueError(f"Layer {layer_idx} not initialized")
        return lay.attend(query)

    def attend_fused(self, layer_idx: int, query: torch.Tensor) -> torch.Tensor:
        return self.attend(layer_idx, query)

    def memory_bytes(self) -> dict:
        tot = {"near": 0, "far": 0, "archive": 0}
        for lay in self.layers:
            if lay is None:
                continue
            m = lay.memory_bytes()
            for key in tot:
                tot[key] += m[key]
        tot["total_quantized"] = tot["near"] + tot["far"]
        tot["total_with_archive"] = tot["total_quantized"] + tot["archive"]
        return tot


MLXFoveatedLayer = FoveatedLayer
MLXFoveatedKVCache = FoveatedKVCache
