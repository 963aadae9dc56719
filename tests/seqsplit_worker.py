"""torchrun worker for test_nccl_seqsplit_two_gpus: each rank tiers its shard
of a seeded prefill, decodes through NCCL all-gather + combine, and rank 0
compares with the unsplit single-GPU fused decode."""
import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
from foveated_kv_b200 import TierConfig, compress_layer  # noqa: E402
from foveated_kv_b200.seqsplit import (shard_bounds, compress_shard, decode_seqsplit,  # noqa: E402
                                       SeqSplitDecoder)
from foveated_kv_b200.synthetic import numpy_workload  # noqa: E402


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(int(os.environ["LOCAL_RANK"]))
    dev = torch.device("cuda", int(os.environ["LOCAL_RANK"]))
    dist.init_process_group("nccl", device_id=dev)
    S, B, Hk, Hq, D = 6000, 1, 2, 8, 128
    w = numpy_workload(13, B, Hk, Hq, S, D, 0)
    t = {k: torch.from_numpy(v).to(dev) for k, v in w.items()}
    cfg = TierConfig(near_pct=0.05, window_size=32, spike_margin=0.5)
    lo, hi = shard_bounds(S, rank, world)
    lay, off = compress_shard(t["k"][:, :, lo:hi], t["v"][:, :, lo:hi], S, lo, cfg)
    out, fl, tk = decode_seqsplit(lay, t["q"], off)
    dec = SeqSplitDecoder(lay, off, Hq)
    o2, f2, t2 = dec.step(t["q"])
    o2, f2, t2 = dec.step(t["q"])          # second step re-uses every buffer
    torch.cuda.synchronize()
    assert torch.equal(o2, out) and torch.equal(f2, fl) and torch.equal(t2, tk)
    # peer-store exchange (one fused launch per rank, no NCCL on the step),
    # eager and captured in a CUDA graph, several steps in a row
    pdec = SeqSplitDecoder(lay, off, Hq, exchange="peer")
    for _ in range(3):
        o3, f3, t3 = pdec.step(t["q"])
        torch.cuda.synchronize()
        assert torch.equal(o3, out) and torch.equal(f3, fl) and torch.equal(t3, tk)
    gs = torch.cuda.Stream(dev)
    gs.wait_stream(torch.cuda.current_stream())
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=gs):
        pdec.step(t["q"])
    for _ in range(4):
        pdec.out.zero_()
        g.replay()
        torch.cuda.synchronize()
        assert torch.equal(pdec.out.view_as(out), out)
        assert torch.equal(pdec.flags.view_as(fl), fl) and torch.equal(pdec.tokens.view_as(tk), tk)
    assert pdec.peer.status() == 0
    dist.barrier()
    pdec.peer.close()
    if rank == 0:
        full = compress_layer(t["k"], t["v"], cfg)
        ro, rf, rt = full.attend_fused_with_spikes(t["q"])
        err = (out.float() - ro.float()).abs().max().item()
        assert err < 2e-3, err
        assert torch.equal(fl, rf) and torch.equal(tk, rt)
        print("SEQSPLIT_OK", err, flush=True)
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
