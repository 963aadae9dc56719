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
    st = pipe.get_stats()
    assert st["spikes_detected"] > 0 and st["promotions_completed"] == total
    pipe.close()


class RecordingAttention(TinyAttention):
    """TinyAttention that keeps the query and output of its decode-time
    attention call (the call the closure routes to the fused kernel)."""

    def forward(self, x, cache):
        B, T, _ = x.shape
        q = (x @ self.wq).view(B, T, self.Hq, self.D).transpose(1, 2)
        k = (x @ self.wk).view(B, T, self.Hk, self.D).transpose(1, 2)
        v = (x @ self.wv).view(B, T, self.Hk, self.D).transpose(1, 2)
        k, v = cache.update_and_fetch(k, v)
        rep = self.Hq // self.Hk
        o = F.scaled_dot_product_attention(q, k.repeat_interleave(rep, 1),
                                           v.repeat_interleave(rep, 1), is_causal=T > 1)
        if T == 1:
            self.last_q, self.last_o = q.detach().clone(), o.detach().clone()
        return o.transpose(1, 2).reshape(B, T, -1) @ self.wo


@pytest.mark.gpu
def test_decode_steps_match_oracle_per_layer():
    """L-layer decode steps through the closure (mlx_generate.py:266-386):
    every layer's attention output in every step equals the oracle's
    dequantise-then-attend over that layer's tiers at that moment -- valid
    near rows including the rows promoted after earlier steps, the far tier,
    and the decode buffer holding this step's token -- within the parity
    tolerance; spikes are drained and promoted between steps."""
    from oracle import fkv_oracle as O
    from tests.helpers import np_, layer_to_oracle, assert_output_close, assert_spikes_match
    torch.manual_seed(0)
    dev = "cuda"
    d_model, Hq, Hk, D, L = 128, 8, 2, 128, 3
    layers = [RecordingAttention(d_model, Hq, Hk, D, 20 + i).to(dev).half() for i in range(L)]
    x = torch.randn(2, 700, d_model, device=dev, dtype=torch.float16)
    fov = FoveatedKVCache(TierConfig(window_size=16, near_pct=0.1, spike_margin=0.0))
    h = x
    with torch.no_grad():
        for i, lay in enumerate(layers):
            h = h + lay(h, PrefillCache(fov, i))
    fov.compress()
    wrappers = G.install_fused_attention(None, fov)
    pipe = PromotionPipeline(L, cooldown_steps=0, max_per_drain=16)
    for i, lay in enumerate(fov.layers):
        pipe.register_archive_host(i, lay.archive_k.cpu(), lay.archive_v.cpu(), lay.far_idx)
        pipe.register_blob(i, lay.get_blob_info())
    nv0 = [np_(l.near_valid).copy() for l in fov.layers]
    tok = h[:, -1:]
    with torch.no_grad():
        for step in range(5):
            hh = tok
            for i, lay in enumerate(layers):
                hh = hh + lay(hh, wrappers[i])
            torch.cuda.synchronize()
            for i, lay in enumerate(layers):
                fl_ = fov.layers[i]
                q = np_(lay.last_q[:, :, 0])
                dk, dv = np_(fl_.decode_k), np_(fl_.decode_v)
                rout, rfl, rtk, diag = O.decode_attend(layer_to_oracle(fl_), q, dk, dv, 0.0)
                assert_output_close(np_(lay.last_o[:, :, 0]).astype(np.float64), rout,
                                    f"step {step} layer {i}")
                w = wrappers[i]
                # identical except decisions inside the numerical tie band
                assert_spikes_match(np_(w._spike_flags), np_(w._spike_tokens), rfl, rtk, diag, 0.0)
            tok = hh
            G.drain_spikes(wrappers, pipe, step)
            pipe.flush()
    torch.cuda.synchronize()
    grown = sum(int((np_(l.near_valid) - n0).sum()) for l, n0 in zip(fov.layers, nv0))
    assert grown > 0 and grown == pipe.get_stats()["promotions_completed"]
    pipe.close()


@pytest.mark.gpu
def test_l_layer_decode_step_in_one_cuda_graph():
    """All L layers' fused decode calls of a step captured in one CUDA graph
    (fixed query buffers, one launch per layer) replay to the same outputs,
    flags and tokens as the eager calls."""
    from foveated_kv_b200 import compress_layer
    from foveated_kv_b200.synthetic import torch_workload
    L, B, Hk, Hq, S, D = 4, 2, 4, 16, 3000, 128
    lays, qs = [], []
    for i in range(L):
        w = torch_workload(50 + i, B, Hk, Hq, S, D, 3, "cuda")
        lay = compress_layer(w["k"], w["v"], TierConfig(spike_margin=0.5))
        for j in range(3):
            lay.add_token(w["dec_k"][:, :, j:j + 1], w["dec_v"][:, :, j:j + 1])
        lays.append(lay)
        qs.append(w["q"].clone())
    eager = [tuple(t.clone() for t in l.attend_fused_with_spikes(q)) for l, q in zip(lays, qs)]
    outs = [torch.empty_like(e[0]) for e in eager]
    res = [None] * L
    st = torch.cuda.Stream()
    st.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(st):
        for i in range(L):                 # warm-up on the capture stream
            lays[i].attend_fused_with_spikes(qs[i], out=outs[i])
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=st):
        for i in range(L):
            res[i] = lays[i].attend_fused_with_spikes(qs[i], out=outs[i])
    for _ in range(3):
        for o in outs:
            o.zero_()
        g.replay()
        torch.cuda.synchronize()
        for i in range(L):
            assert torch.equal(res[i][0], eager[i][0])
            assert torch.equal(res[i][1], eager[i][1]) and torch.equal(res[i][2], eager[i][2])
