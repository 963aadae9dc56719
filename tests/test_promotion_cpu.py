"""Promotion pipeline host logic (no GPU): the C++ drain filter against the
oracle's restatement of PromotionPipeline::drain_spikes, the disk archive
format, and injected failures (missing / truncated archive files)."""

import numpy as np
import pytest
import torch

from oracle.fkv_oracle import DrainFilter
from foveated_kv_b200 import PromotionPipeline, create_disk_archive, FkvNativeError


def _archive(B, H, S, D, seed=0):
    rs = np.random.RandomState(seed)
    k = rs.standard_normal((B, H, S, D)).astype(np.float16)
    v = rs.standard_normal((B, H, S, D)).astype(np.float16)
    idx = np.broadcast_to(np.arange(100, 100 + S, dtype=np.int32), (B, H, S)).copy()
    return k, v, idx


@pytest.mark.parametrize("B,Hq,Hk,budget,cool", [(1, 32, 8, 8, 5), (3, 8, 2, 4, 2), (2, 4, 4, 100, 0)])
def test_drain_filter_matches_oracle(B, Hq, Hk, budget, cool):
    S, D, L = 50, 16, 2
    k, v, idx = _archive(B, Hk, S, D)
    pipe = PromotionPipeline(L, cooldown_steps=cool, max_per_drain=budget, device=0)
    ref = DrainFilter(cool, budget)
    for layer in range(L):
        pipe.register_archive_host(layer, k, v, idx)
    rs = np.random.RandomState(1)
    for step in range(12):
        for layer in range(L):
            flags = (rs.rand(B, Hq) < 0.4).astype(np.int32)
            toks = rs.randint(-1, S + 2, size=(B, Hq)).astype(np.int32)   # includes invalid
            n = pipe.drain_spikes(layer, flags, toks, idx, step)
            exp = ref.drain(layer, flags, toks, idx, step, arc_len=S)
            assert n == len(exp)
    st = pipe.get_stats()
    assert st["spikes_detected"] == ref.stats["spikes_detected"]
    assert st["spikes_queued"] == ref.stats["spikes_queued"]
    assert st["spikes_deduplicated"] == ref.stats["spikes_deduplicated"]
    assert st["spikes_cooled_down"] == ref.stats["spikes_cooled_down"]
    pipe.stop()
    pipe.close()


def test_drain_without_archive_is_noop():
    pipe = PromotionPipeline(1, device=0)
    flags = np.ones((1, 4), np.int32)
    assert pipe.drain_spikes(0, flags, np.zeros((1, 4), np.int32), np.zeros((1, 4, 5), np.int32), 0) == 0
    assert pipe.get_stats()["spikes_detected"] == 0
    pipe.close()


def test_bad_layer_raises():
    pipe = PromotionPipeline(2, device=0)
    with pytest.raises(FkvNativeError):
        pipe.drain_spikes(5, np.zeros((1, 1), np.int32), np.zeros((1, 1), np.int32),
                          np.zeros((1, 1, 1), np.int32), 0)
    pipe.close()


def test_disk_archive_roundtrip_bit_exact(tmp_path):
    # reference tests/test_disk_archive.py:25-69
    k, v, idx = _archive(1, 2, 64, 64)
    arc = create_disk_archive(torch.from_numpy(k), torch.from_numpy(v), torch.from_numpy(idx),
                              0, tmp_path)
    pk, pv = arc.promote(head=0, archive_local_idx=10)
    assert pk.shape == (1, 1, 1, 64)
    assert np.array_equal(pk.numpy()[0, 0, 0].view(np.uint16), k[0, 0, 10].view(np.uint16))
    assert np.array_equal(pv.numpy()[0, 0, 0].view(np.uint16), v[0, 0, 10].view(np.uint16))
    bk, bv = arc.promote_batch(head=1, archive_local_indices=[5, 10, 20])
    assert np.array_equal(bk.numpy()[0, 0], k[0, 1, [5, 10, 20]])
    assert arc.disk_bytes() == 2 * 64 * 64 * 2 * 2
    assert (tmp_path / "archive_k_layer0.bin").stat().st_size == 2 * 64 * 64 * 2
    assert create_disk_archive(torch.zeros(1, 2, 0, 64), torch.zeros(1, 2, 0, 64),
                               torch.zeros(1, 2, 0, dtype=torch.int32), 1, tmp_path) is None


def test_disk_archive_registers_and_drains(tmp_path):
    k, v, idx = _archive(1, 2, 30, 32)
    arc = create_disk_archive(torch.from_numpy(k), torch.from_numpy(v), torch.from_numpy(idx),
                              3, tmp_path)
    pipe = PromotionPipeline(4, device=0)
    pipe.register_archive(3, arc.path_k, arc.path_v, 2, 30, 32, idx)
    n = pipe.drain_spikes(3, np.array([[1, 0, 0, 1]], np.int32), np.array([[3, 0, 0, 7]], np.int32),
                          idx, 0)
    assert n == 2
    pipe.close()


def test_missing_and_truncated_archive_fail_loudly(tmp_path):
    pipe = PromotionPipeline(1, device=0)
    idx = np.zeros((1, 2, 8), np.int32)
    with pytest.raises(FkvNativeError, match="I/O"):
        pipe.register_archive(0, str(tmp_path / "nope_k.bin"), str(tmp_path / "nope_v.bin"),
                              2, 8, 16, idx)
    short = tmp_path / "short.bin"
    short.write_bytes(b"\0" * 100)          # needs 2*8*16*2 = 512 bytes
    with pytest.raises(FkvNativeError, match="I/O"):
        pipe.register_archive(0, str(short), str(short), 2, 8, 16, idx)
    with pytest.raises(FkvNativeError):
        pipe.register_archive(0, str(short), str(short), 2, 8, 16, idx[:, :, :4])   # idx too short
    pipe.close()
