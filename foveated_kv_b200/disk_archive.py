"""Disk-backed fp16 archive (mirror of src/foveated_kv/disk_archive.py).

Layout per layer: ``archive_k_layer{L}.bin`` and ``archive_v_layer{L}.bin``,
flat fp16 of shape (B, H_kv, S_arc, D) row-major; with B = 1 this is the
reference's (H_kv, S_arc, D) format.  The promotion pipeline maps these files
(fkv_promo_register_archive); DiskArchive reads them with numpy.memmap.
"""

from __future__ import annotations

from dataclasses import dataclass
from pathlib import Path
from typing import Union

import numpy as np
import torch


@dataclass
class DiskArchive:
    path_k: str
    path_v: str
    mmap_k: np.memmap   # (B, H_kv, S_arc, D) fp16
    mmap_v: np.memmap
    idx: torch.Tensor   # (B, H_kv, S_arc) int32 positions
    B: int
    H_kv: int
    S_arc: int
    D: int

    def promote(self, head: int, archive_local_idx: int, b: int = 0):
        """Exact fp16 K, V of one archived token as (1, 1, 1, D) tensors."""
        k = torch.from_numpy(np.array(self.mmap_k[b, head, archive_local_idx]))
        v = torch.from_numpy(np.array(self.mmap_v[b, head, archive_local_idx]))
        return k.reshape(1, 1, 1, self.D), v.reshape(1, 1, 1, self.D)

    def promote_batch(self, head: int, archive_local_indices, b: int = 0):
        n = len(archive_local_indices)
        if n == 0:
            z = torch.zeros((1, 1, 0, self.D), dtype=torch.float16)
            return z, z.clone()
        ix = np.asarray(archive_local_indices)
        k = torch.from_numpy(np.array(self.mmap_k[b, head, ix]))
        v = torch.from_numpy(np.array(self.mmap_v[b, head, ix]))
        return k.reshape(1, 1, n, self.D), v.reshape(1, 1, n, self.D)

    def score_boundary_tokens(self, head: int, query, token_indices, b: int = 0) -> np.ndarray:
        """Scores k . q of archived tokens for host-side rescoring
        (disk_archive.py:89-109): (N,) float32."""
        if len(token_indices) == 0:
            return np.array([], dtype=np.float32)
        k = np.asarray(self.mmap_k[b, head, np.asarray(token_indices)], dtype=np.float32)
        return k @ np.asarray(query, dtype=np.float32)

    def memory_bytes_in_ram(self) -> int:
        return self.idx.numel() * self.idx.element_size()

    def disk_bytes(self) -> int:
        return self.B * self.H_kv * self.S_arc * self.D * 2 * 2

    def close(self):
        del self.mmap_k
        del self.mmap_v


def create_disk_archive(archive_k: torch.Tensor, archive_v: torch.Tensor,
                        archive_idx: torch.Tensor, layer_idx: int,
                        archive_dir: Union[str, Path]):
    """Write one layer's archive to disk (create_disk_archive,
    disk_archive.py:127-185); returns None when the layer has no far tokens."""
    d = Path(archive_dir)
    d.mkdir(parents=True, exist_ok=True)
    B, H, S, D = archive_k.shape
    if S == 0:
        return None
    pk = str(d / f"archive_k_layer{layer_idx}.bin")
    pv = str(d / f"archive_v_layer{layer_idx}.bin")
    archive_k.detach().to(torch.float16).cpu().contiguous().numpy().tofile(pk)
    archive_v.detach().to(torch.float16).cpu().contiguous().numpy().tofile(pv)
    mk = np.memmap(pk, dtype=np.float16, mode="r", shape=(B, H, S, D))
    mv = np.memmap(pv, dtype=np.float16, mode="r", shape=(B, H, S, D))
    return DiskArchive(pk, pv, mk, mv, archive_idx.detach().cpu(), B, H, S, D)


def offload_cache_to_disk(cache, archive_dir: Union[str, Path]) -> list:
    """Move every layer's device archive to disk (offload_cache_to_disk,
    disk_archive.py:188-222), freeing the device copies."""
    out = []
    for i, lay in enumerate(cache.layers):
        if lay is None or lay.archive_k is None:
            out.append(None)
            continue
        out.append(create_disk_archive(lay.archive_k, lay.archive_v, lay.archive_idx, i,
                                       archive_dir))
        lay.archive_k = None
        lay.archive_v = None
    return out
