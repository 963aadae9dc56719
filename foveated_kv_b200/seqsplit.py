"""Sequence-split decode across GPUs (long contexts; no reference counterpart:
the reference has no multi-device code).

The prefill sequence [0, S) is split into world_size contiguous shards of
positions (``shard_bounds``: equal length; ``shard_bounds_balanced``: equal
decode cost).  Each rank tiers its shard with the GLOBAL recency tier boundaries
(a position is near or far exactly as in the unsplit cache), runs the fused
decode kernel in partial mode (one (m, l, o, min_near, max_far, argmax)
record per (b, q head), argmax as a global far index), all-gathers the
records over NCCL (NVLink), and merges them with fkv_combine_partials in
rank order, so flags / tokens equal those of the unsplit cache.  The decode
buffer lives on the last rank (it holds the sequence's tail).
"""

from __future__ import annotations

import ctypes as C
from typing import Optional

import numpy as np
import torch
import torch.distributed as dist

from . import _native
from .cache import FoveatedLayer, _Workspace, _p, _stream, F16, I32, U8
from .config import TierConfig


def shard_bounds(S: int, rank: int, world: int):
    """Even split of [0, S): shard `rank` is [lo, hi)."""
    base, rem = divmod(S, world)
    lo = rank * base + min(rank, rem)
    return lo, lo + base + (1 if rank < rem else 0)


def shard_bounds_balanced(S: int, rank: int, world: int, cfg: TierConfig):
    """Split [0, S) into `world` contiguous shards of equal decode cost: an
    fp16 near token costs 2 (K+V at 2 bytes/element), a compressed far token
    1.  The global near tier (sinks, recent middle, window) sits at the two
    ends of the sequence, so equal-length shards leave the last rank with most
    of the fp16 rows."""
    if world == 1:
        return 0, S
    tb = cfg.tier_boundaries(S)
    cost = np.ones(S, dtype=np.int64)
    cost[:tb["n_sinks"]] = 2
    cost[tb["near_mid_start"]:] = 2
    cum = np.concatenate([[0], np.cumsum(cost)])
    cuts = [0] + [int(np.searchsorted(cum, cum[-1] * r / world)) for r in range(1, world)] + [S]
    return cuts[rank], cuts[rank + 1]


def _shard_ranges(S: int, lo: int, hi: int, tb: dict):
    """Global-tier near ranges (sinks, recent middle, window) and the far range,
    each clipped to the shard [lo, hi), as (a, b) pairs."""
    ns, w, ms, me, nms = tb["n_sinks"], tb["window"], tb["mid_start"], tb["mid_end"], tb["near_mid_start"]
    clip = lambda a, b: (max(a, lo), max(min(b, hi), max(a, lo)))
    return [clip(0, ns), clip(nms, me), clip(S - w, S)], clip(ms, nms)


def shard_positions(S: int, lo: int, hi: int, cfg: TierConfig):
    """Global-tier near / far positions inside [lo, hi) and the global far
    index of the shard's first far token."""
    tb = cfg.tier_boundaries(S)
    near_r, (fa, fb) = _shard_ranges(S, lo, hi, tb)
    near = np.concatenate([np.arange(a, b, dtype=np.int32) for a, b in near_r])
    far = np.arange(fa, fb, dtype=np.int32)
    off = int(far[0] - tb["mid_start"]) if far.size else 0
    return near, far, off, tb


def compress_shard(k_shard: torch.Tensor, v_shard: torch.Tensor, S: int, lo: int,
                   cfg: TierConfig, keep_archive: bool = False) -> tuple:
    """Tier one rank's shard (B, H, hi-lo, D) of a length-S prefill.
    Returns (FoveatedLayer, far_index_offset)."""
    lib = _native.load()
    k = k_shard.to(F16).contiguous()
    v = v_shard.to(F16).contiguous()
    B, H, Ssh, D = k.shape
    dev = k.device
    tb = cfg.tier_boundaries(S)
    near_r, (fa, fb) = _shard_ranges(S, lo, lo + Ssh, tb)
    # index lists built on the device (no host arrays, no host->device copies)
    near = torch.cat([torch.arange(a - lo, b - lo, dtype=I32, device=dev) for a, b in near_r])
    R = int(near.numel())
    Np = R + max(int(R * cfg.promo_headroom_pct), cfg.promo_headroom_min)
    Fn = fb - fa
    off = fa - tb["mid_start"] if Fn > 0 else 0
    L = _native.TierLayout()
    L.S, L.n_near_padded, L.far_count, L.r_actual = Ssh, Np, Fn, R
    near_idx = torch.full((B, H, Np), -1, dtype=I32, device=dev)
    near_idx[:, :, :R] = near
    far_idx_local = torch.arange(fa - lo, fb - lo, dtype=I32, device=dev).expand(B, H, Fn).contiguous()
    near_k = torch.empty((B, H, Np, D), dtype=F16, device=dev)
    near_v = torch.empty_like(near_k)
    far_k = torch.empty((B, H, Fn, D), dtype=U8, device=dev)
    far_v = torch.empty((B, H, Fn, D // 2), dtype=U8, device=dev)
    vg = cfg.v_group
    sshape = (B, H, Fn) if vg is None else (B, H, Fn, D // vg)
    vsc = torch.empty(sshape, dtype=F16, device=dev)
    vze = torch.empty(sshape, dtype=F16, device=dev)
    arc_k = torch.empty((B, H, Fn, D), dtype=F16, device=dev) if keep_archive else None
    arc_v = torch.empty_like(arc_k) if keep_archive else None
    _native.check(lib.fkv_compress_fp8(
        C.byref(L), B, H, D, _p(k), _p(v), Ssh * D, _p(near_idx), _p(far_idx_local),
        int(vg or 0), _p(near_k), _p(near_v), _p(far_k), _p(far_v), _p(vsc), _p(vze),
        _p(arc_k), _p(arc_v), _stream(dev)), "fkv_compress_fp8")
    near_idx[:, :, :R] += lo
    lay = FoveatedLayer(near_k=near_k, near_v=near_v, near_idx=near_idx,
                        near_valid=torch.full((B, H), R, dtype=I32, device=dev),
                        far_idx=(far_idx_local + lo), archive_k=arc_k, archive_v=arc_v,
                        far_k=far_k, far_v=far_v, far_v_scale=vsc, far_v_zero=vze,
                        v_group=vg, spike_margin=cfg.spike_margin)
    return lay, off


def decode_partial(layer: FoveatedLayer, q: torch.Tensor, far_offset: int):
    """This shard's partial records: part (B*Hq, D+4) f32, arg (B*Hq) int32.
    Both are views of one flat f32 buffer (arg bit-cast), so a single
    collective can exchange them."""
    lib = _native.load()
    if not (q.is_cuda and layer.near_k.is_cuda):
        raise ValueError("decode_partial: query and tiers must be CUDA tensors")
    B, Hq, D = q.shape[0], q.shape[1], q.shape[-1]
    qq = q.reshape(B, Hq, D).to(F16).contiguous()
    sh = layer._fill_shape(Hq, layer.spike_margin)
    ws = _Workspace.get(lib.fkv_decode_workspace_bytes(C.byref(sh)), layer.device)
    N = B * Hq
    flat = torch.empty((N * (D + 4) + N,), dtype=torch.float32, device=layer.device)
    part = flat[:N * (D + 4)].view(N, D + 4)
    arg = flat[N * (D + 4):].view(torch.int32)
    dk = layer._dec_k if layer.n_decode else None
    dv = layer._dec_v if layer.n_decode else None
    _native.check(lib.fkv_decode_fp8_partial(
        C.byref(sh), _p(layer.near_k), _p(layer.near_v), _p(layer.near_valid), _p(layer.far_k),
        _p(layer.far_v), _p(layer.far_v_scale), _p(layer.far_v_zero), _p(qq), _p(dk), _p(dv),
        int(far_offset), _p(part), _p(arg), ws.data_ptr(), ws.numel(), _stream(layer.device)),
        "fkv_decode_fp8_partial")
    return part, arg


def _joined_view(part: torch.Tensor, arg: torch.Tensor):
    """The flat [records | argmax] buffer when part and arg are the two views
    decode_partial makes of it, else None."""
    N, D4 = part.shape
    if arg.dtype != torch.int32 or arg.numel() != N or not part.is_contiguous():
        return None
    if part.data_ptr() + N * D4 * 4 != arg.data_ptr():
        return None
    if part.untyped_storage().data_ptr() != arg.untyped_storage().data_ptr():
        return None
    if part.untyped_storage().nbytes() < part.storage_offset() * 4 + (N * D4 + N) * 4:
        return None
    return torch.empty((0,), dtype=torch.float32, device=part.device).set_(
        part.untyped_storage(), part.storage_offset(), (N * D4 + N,), (1,))


def gather_partials(part: torch.Tensor, arg: torch.Tensor, group=None):
    """All-gather every rank's records: (P, N, D+4) and (P, N), rank order.
    One collective when part and arg share one buffer (as decode_partial
    returns them), two otherwise; NCCL over NVLink on GPUs, any backend works
    (gloo for host tests)."""
    if not (dist.is_available() and dist.is_initialized()):
        return part[None], arg[None]          # single process: nothing to exchange
    P = dist.get_world_size(group)
    N, D4 = part.shape
    flat = _joined_view(part, arg)
    if flat is not None:
        out = torch.empty((P * (N * D4 + N),), dtype=torch.float32, device=part.device)
        dist.all_gather_into_tensor(out, flat, group=group)
        out = out.view(P, N * D4 + N)
        return (out[:, :N * D4].contiguous().view(P, N, D4),
                out[:, N * D4:].contiguous().view(torch.int32))
    parts = torch.empty((P * N, D4), dtype=part.dtype, device=part.device)
    args = torch.empty((P * arg.shape[0],), dtype=arg.dtype, device=arg.device)
    dist.all_gather_into_tensor(parts, part.contiguous(), group=group)
    dist.all_gather_into_tensor(args, arg.contiguous(), group=group)
    return parts.view(P, N, D4), args.view(P, -1)


def combine(parts: torch.Tensor, args: torch.Tensor, margin: float):
    """Merge (P, N, D+4) records on the device: out (N, D) fp16, flags, tokens."""
    lib = _native.load()
    parts, args = parts.contiguous(), args.contiguous()   # the C ABI reads dense arrays
    P, N, D4 = parts.shape
    D = D4 - 4
    out = torch.empty((N, D), dtype=F16, device=parts.device)
    flags = torch.empty((N,), dtype=I32, device=parts.device)
    tokens = torch.empty((N,), dtype=I32, device=parts.device)
    _native.check(lib.fkv_combine_partials(P, N, D, _p(parts), _p(args), float(margin), _p(out),
                                           _p(flags), _p(tokens), _stream(parts.device)),
                  "fkv_combine_partials")
    return out, flags, tokens


def decode_seqsplit(layer: FoveatedLayer, q: torch.Tensor, far_offset: int, group=None):
    """One decode step of a sequence-split layer: local partial, all-gather,
    combine.  Returns (out (B, Hq, 1, D), flags (B, Hq), tokens (B, Hq))."""
    B, Hq, D = q.shape[0], q.shape[1], q.shape[-1]
    part, arg = decode_partial(layer, q, far_offset)
    parts, args = gather_partials(part, arg, group)
    out, fl, tk = combine(parts, args, layer.spike_margin)
    return out.view(B, Hq, 1, D), fl.view(B, Hq), tk.view(B, Hq)


class SeqSplitDecoder:
    """Repeated sequence-split decode steps of one layer shard.

    The decode shape, a workspace, the [records | argmax] buffer, the buffer
    that receives every rank's copy of it and the outputs are prepared once;
    a step is then one partial-kernel call, one all-gather and one combine
    call that reads the gathered blocks in place
    (fkv_combine_partials_strided).  Little host work per step matters when
    several ranks share a host's cores.  The tensors step() returns are
    overwritten by the next step: copy them to keep them."""

    def __init__(self, layer: FoveatedLayer, far_offset: int, Hq: int, group=None,
                 exchange: str = "nccl"):
        """exchange: 'nccl' (all-gather + strided merge) or 'peer' (one
        fused peer-store exchange + merge launch, PeerExchange)."""
        self.lib = _native.load()
        self.layer, self.far_offset, self.group = layer, int(far_offset), group
        self.P = dist.get_world_size(group) if (dist.is_available() and dist.is_initialized()) else 1
        self.B, self.Hq, self.D = layer.B, Hq, layer.D
        self.N = self.B * Hq
        self.rec = self.N * (self.D + 4) + self.N          # floats per rank block
        dev = layer.device
        self.sh = _native.DecodeShape()
        self.ws = None
        self._refresh_shape()
        self.peer = None
        if exchange == "peer" and self.P > 1:
            self.peer = PeerExchange(self.N, self.D, dev, group)
            self.flat = torch.zeros((self.peer.stride,), dtype=torch.float32, device=dev)
            self.gathered = self.flat
        else:
            self.flat = torch.empty((self.rec,), dtype=torch.float32, device=dev)
            self.gathered = (torch.empty((self.P * self.rec,), dtype=torch.float32, device=dev)
                             if self.P > 1 else self.flat)
        self.qbuf = torch.empty((self.B, Hq, self.D), dtype=F16, device=dev)
        self.out = torch.empty((self.N, self.D), dtype=F16, device=dev)
        self.flags = torch.empty((self.N,), dtype=I32, device=dev)
        self.tokens = torch.empty((self.N,), dtype=I32, device=dev)

    def _refresh_shape(self):
        src = self.layer._fill_shape(self.Hq, self.layer.spike_margin)
        key = (src.n_dec, src.dec_stride)
        C.memmove(C.addressof(self.sh), C.addressof(src), C.sizeof(self.sh))
        if self.ws is None or key != self._ws_key:
            need = self.lib.fkv_decode_workspace_bytes(C.byref(self.sh)) + 256
            if self.ws is None or self.ws.numel() < need:
                self.ws = torch.zeros((need,), dtype=torch.uint8, device=self.layer.device)
            self._ws_key = key

    def step(self, q: torch.Tensor):
        """One decode step: returns (out (B, Hq, 1, D), flags (B, Hq), tokens (B, Hq))."""
        lay, lib, N, D = self.layer, self.lib, self.N, self.D
        if (lay._n_dec, lay._dec_k.shape[2]) != self._ws_key:
            self._refresh_shape()
        qq = q.reshape(self.B, self.Hq, D)
        if qq.dtype != F16 or not qq.is_contiguous():
            self.qbuf.copy_(qq)
            qq = self.qbuf
        dk = lay._dec_k if lay.n_decode else None
        dv = lay._dec_v if lay.n_decode else None
        st = _stream(lay.device)
        base = self.flat.data_ptr()
        _native.check(lib.fkv_decode_fp8_partial(
            C.byref(self.sh), _p(lay.near_k), _p(lay.near_v), _p(lay.near_valid), _p(lay.far_k),
            _p(lay.far_v), _p(lay.far_v_scale), _p(lay.far_v_zero), _p(qq), _p(dk), _p(dv),
            self.far_offset, base, base + N * (D + 4) * 4, self.ws.data_ptr(), self.ws.numel(), st),
            "fkv_decode_fp8_partial")
        if self.peer is not None:
            self.peer.combine(self.flat, lay.spike_margin, self.out, self.flags, self.tokens)
            return (self.out.view(self.B, self.Hq, 1, D), self.flags.view(self.B, self.Hq),
                    self.tokens.view(self.B, self.Hq))
        if self.P > 1:
            dist.all_gather_into_tensor(self.gathered, self.flat, group=self.group)
        g = self.gathered.data_ptr()
        _native.check(lib.fkv_combine_partials_strided(
            self.P, N, D, g, self.rec, g + N * (D + 4) * 4, self.rec, float(lay.spike_margin),
            self.out.data_ptr(), self.flags.data_ptr(), self.tokens.data_ptr(), st),
            "fkv_combine_partials_strided")
        return (self.out.view(self.B, self.Hq, 1, D), self.flags.view(self.B, self.Hq),
                self.tokens.view(self.B, self.Hq))


class PeerExchange:
    """Receive buffers of a sequence split mapped into every rank (CUDA IPC
    over NVLink), for fkv_exchange_combine: one launch per rank that writes
    its record block into every peer's buffer with plain peer stores and
    merges once all P blocks of the step have arrived (bounded wait).  No
    NCCL call on the step's path, so the whole step can be captured in a
    CUDA graph.  One rank per GPU; the handles are exchanged once through the
    process group."""

    def __init__(self, N: int, D: int, device, group=None):
        self.lib = lib = _native.load()
        self.P = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.N, self.D = N, D
        self.stride = int(lib.fkv_exchange_block_stride(N, D))
        nbytes = int(lib.fkv_exchange_recv_bytes(self.P, N, D))
        self.recv = torch.zeros((nbytes // 4 + 16,), dtype=torch.float32, device=device)
        base = self.recv.data_ptr()
        self.recv_ptr = (base + 63) & ~63
        self.state = torch.zeros((4,), dtype=I32, device=device)
        hb = lib.fkv_ipc_handle_bytes()
        handle = (C.c_uint8 * hb)()
        off = C.c_int64(0)
        _native.check(lib.fkv_ipc_get_handle(self.recv_ptr, handle, C.byref(off)), "fkv_ipc_get_handle")
        mine = (bytes(handle), int(off.value))
        allh = [None] * self.P
        dist.all_gather_object(allh, mine, group=group)
        self.opened = []
        ptrs = []
        for r, (h, o) in enumerate(allh):
            if r == self.rank:
                ptrs.append(self.recv_ptr)
                continue
            out = C.c_void_p()
            hbuf = (C.c_uint8 * hb).from_buffer_copy(h)
            _native.check(lib.fkv_ipc_open(hbuf, o, C.byref(out)), "fkv_ipc_open")
            self.opened.append((out.value, o))
            ptrs.append(out.value)
        self.peers = torch.tensor(ptrs, dtype=torch.int64, device=device)
        torch.cuda.synchronize(device)
        dist.barrier(group=group)       # every rank's buffers are mapped before any step

    def combine(self, local_block: torch.Tensor, margin: float, out, flags, tokens):
        _native.check(self.lib.fkv_exchange_combine(
            self.P, self.rank, self.N, self.D, local_block.data_ptr(), self.peers.data_ptr(),
            self.recv_ptr, self.state.data_ptr(), float(margin), out.data_ptr(), flags.data_ptr(),
            tokens.data_ptr(), _stream(local_block.device)), "fkv_exchange_combine")

    def status(self) -> int:
        """FKV_ERR_TIMEOUT (-4) if a peer's block did not arrive in some step."""
        return int(self.state[3].item())

    def close(self):
        for ptr, off in self.opened:
            self.lib.fkv_ipc_close(ptr, off)
        self.opened = []
