"""Decode-time integration with torch models (mirror of
src/foveated_kv/mlx_generate.py:42-259).

``install_fused_sdpa`` replaces ``torch.nn.functional.scaled_dot_product_attention``
with a closure: prefill calls (query length > 1) go to the original SDPA;
decode calls (query length 1) are routed, by a rolling layer counter, to
``FoveatedLayer.attend_fused_with_spikes`` and return its output, stashing the
per-head spike flags/tokens on the layer's ``FusedCacheWrapper``.
``drain_spikes`` resets the counter after a decode step and feeds the spikes
to a PromotionPipeline.
"""

from __future__ import annotations

from typing import Optional

import torch
import torch.nn.functional as F

from .cache import FoveatedKVCache, FoveatedLayer


class _FusedSDPAState:
    original_sdpa = None
    installed: bool = False
    fov_cache: Optional[FoveatedKVCache] = None
    layer_counter: int = 0
    n_layers: int = 0
    decode_step: int = 0
    wrappers: Optional[list] = None
    disabled: bool = False
    pipeline = None


_state = _FusedSDPAState()


class FusedCacheWrapper:
    """Per-layer cache object handed to the model (mlx_generate.py:57-81): the
    model appends its new K/V through ``update_and_fetch``; attention itself
    runs in the fused kernel through the SDPA closure."""

    def __init__(self, fov_layer: FoveatedLayer, layer_idx: int):
        self.fov_layer = fov_layer
        self.layer_idx = layer_idx
        self.offset = fov_layer.total_tokens
        self._spike_flags = None
        self._spike_tokens = None

    @property
    def state(self):
        return self.fov_layer.near_k, self.fov_layer.near_v

    def update_and_fetch(self, keys: torch.Tensor, values: torch.Tensor):
        self.fov_layer.add_token(keys, values)
        self.offset += keys.shape[2]
        return keys, values


def _build_fused_interceptor(state: _FusedSDPAState):
    original = state.original_sdpa
    layers = state.fov_cache.layers
    n_layers = state.n_layers

    def interceptor(query, key, value, attn_mask=None, dropout_p=0.0, is_causal=False,
                    scale=None, **kwargs):
        if query.dim() != 4 or query.shape[2] > 1:
            return original(query, key, value, attn_mask=attn_mask, dropout_p=dropout_p,
                            is_causal=is_causal, scale=scale, **kwargs)
        idx = state.layer_counter
        state.layer_counter = idx + 1
        if idx >= n_layers:
            idx %= n_layers
        layer = layers[idx]
        if layer is None or state.disabled:
            return original(query, key, value, attn_mask=attn_mask, dropout_p=dropout_p,
                            is_causal=is_causal, scale=scale, **kwargs)
        out, flags, tokens = layer.attend_fused_with_spikes(query)
        ws = state.wrappers
        if ws is not None and idx < len(ws) and ws[idx] is not None:
            ws[idx]._spike_flags = flags
            ws[idx]._spike_tokens = tokens
        return out if out.dtype == query.dtype else out.to(query.dtype)

    return interceptor


def install_fused_sdpa(fov_cache: FoveatedKVCache) -> None:
    """Patch torch.nn.functional.scaled_dot_product_attention (mlx_generate.py:134-158)."""
    if _state.installed:
        raise RuntimeError("Fused SDPA already installed - call uninstall_fused_sdpa() first")
    _state.original_sdpa = F.scaled_dot_product_attention
    _state.fov_cache = fov_cache
    _state.layer_counter = 0
    _state.n_layers = len(fov_cache.layers)
    _state.decode_step = 0
    _state.wrappers = None
    _state.disabled = False
    _state.installed = True
    F.scaled_dot_product_attention = _build_fused_interceptor(_state)


def uninstall_fused_sdpa() -> None:
    if not _state.installed:
        return
    F.scaled_dot_product_attention = _state.original_sdpa
    _state.original_sdpa = None
    _state.fov_cache = None
    _state.layer_counter = 0
    _state.n_layers = 0
    _state.decode_step = 0
    _state.wrappers = None
    _state.disabled = False
    _state.pipeline = None
    _state.installed = False


def install_fused_attention(model, fov_cache: FoveatedKVCache) -> list:
    """Install the closure and return one FusedCacheWrapper per layer
    (mlx_generate.py:184-201)."""
    wrappers = [FusedCacheWrapper(l, i) if l is not None else None
                for i, l in enumerate(fov_cache.layers)]
    install_fused_sdpa(fov_cache)
    _state.wrappers = wrappers
    return wrappers


def uninstall_fused_attention(model=None) -> None:
    uninstall_fused_sdpa()


def set_fused_disabled(flag: bool) -> None:
    """Route every decode call to the original SDPA (the reference's
    ``_fused_disabled``, mlx_generate.py:115-118)."""
    _state.disabled = bool(flag)


def drain_spikes(wrappers: list, pipeline, decode_step: int) -> int:
    """After a decode step: reset the layer counter and drain every layer's
    stashed spikes into ``pipeline`` (mlx_generate.py:209-230).  Returns the
    number of promotions queued."""
    reset_fused_layer_counter()
    if pipeline is None:
        return 0
    n = 0
    for w in wrappers:
        if w is None:
            continue
        if w._spike_flags is not None and w._spike_tokens is not None:
            n += pipeline.drain_spikes(w.layer_idx, w._spike_flags, w._spike_tokens,
                                       w.fov_layer.far_idx, decode_step)
        w._spike_flags = None
        w._spike_tokens = None
    return n


def reset_fused_layer_counter() -> None:
    _state.layer_counter = 0
    _state.decode_step += 1
