"""Tier configuration (mirror of MLXTierConfig, src/foveated_kv/mlx_foveated.py:111-169)."""

from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

from . import _native


@dataclass
class TierConfig:
    """Configuration of the two-tier foveated cache.

    Fields shared with the reference keep its names, defaults and validation
    (mlx_foveated.py:111-126).  Extensions:
      select        'recency' (the reference's behaviour) or 'importance'
                    (sinks + window near, the rest of the near budget to the
                    middle tokens with the highest softmax(q k^T) mass)
      v_group       None = per-token INT4 V scale/zero (the reference), or 32
      spike_margin  margin of the fused kernel's spike test; the reference's
                    live value is 10.0 (mlx_foveated.py:337,355)
      qjl_coef      turbo score-on-codes QJL coefficient: sqrt(pi/2) as the
                    Metal kernel (foveated_attn.metal:518), or 1.0 as the
                    dequant path (turbo_quantize.py:129)
    """

    near_pct: float = 0.10
    n_sinks: int = 4
    window_size: int = 32
    promo_headroom_pct: float = 0.5
    promo_headroom_min: int = 8
    compress_method: str = "fp8"
    select: str = "recency"
    v_group: Optional[int] = None
    spike_margin: float = 10.0
    qjl_coef: float = 1.2533141373155001

    def __post_init__(self):
        if self.compress_method not in ("fp8", "turbo"):
            raise ValueError(
                f"compress_method must be 'fp8' or 'turbo', got '{self.compress_method}'")
        if self.select not in ("recency", "importance"):
            raise ValueError(f"select must be 'recency' or 'importance', got '{self.select}'")
        if self.v_group not in (None, 32):
            raise ValueError(f"v_group must be None or 32, got {self.v_group}")

    def tier_boundaries(self, S: int) -> dict:
        """Tier boundaries for sequence length S (same dict as the reference)."""
        return self.layout(S).as_dict()

    def layout(self, S: int) -> "_native.TierLayout":
        return _native.tier_layout(S, self.near_pct, self.n_sinks, self.window_size,
                                   self.promo_headroom_pct, self.promo_headroom_min)


MLXTierConfig = TierConfig
