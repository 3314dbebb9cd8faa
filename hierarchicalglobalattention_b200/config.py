"""Router hyper-parameters and the hot-window placement policy.

Same fields, defaults and derived quantities as the reference's ``RouterConfig``
(ExistingModelFineTuning/KvRouter/chunk_router.py:58-90) and ``ChunkPlacementPolicy``
(ExistingModelFineTuning/KvRouter/chunk_placement_policy.py:13-38), so configurations and
state_dict-bearing modules built for the reference construct unchanged.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Optional, Tuple

import torch

from . import _lib


@dataclass
class RouterConfig:
    nhead: int
    kv_heads: int
    head_dim: int
    chunk_size: int
    group_size: int
    topk_chunks: int = 20
    topk_groups: int = 32
    current_group_summaries: bool = True
    theta: float = 1_000_000.0
    mixed_rope_threshold: float = 0.5
    mixed_rope_cutoff_pair: Optional[int] = None

    @property
    def groups_per_chunk(self) -> int:
        return self.chunk_size // self.group_size

    @property
    def rep(self) -> int:
        return self.nhead // self.kv_heads

    @property
    def scale(self) -> float:
        return self.head_dim ** -0.5

    @property
    def group_kv_scale(self) -> float:
        return 1.0 / (self.group_size + math.sqrt(self.group_size))

    def hga_params(self, policy: "ChunkPlacementPolicy", batch: int, dtype: torch.dtype) -> _lib.HgaParams:
        """The C-ABI parameter block for this configuration."""
        return _lib.make_params(
            batch=batch, nhead=self.nhead, kv_heads=self.kv_heads, head_dim=self.head_dim,
            chunk_size=self.chunk_size, group_size=self.group_size, topk_chunks=self.topk_chunks,
            topk_groups=self.topk_groups, keep_first=policy.keep_first, keep_last=policy.keep_last,
            theta=self.theta, dtype=dtype, mixed_rope_threshold=self.mixed_rope_threshold,
            mixed_rope_cutoff_pair=self.mixed_rope_cutoff_pair)


@dataclass(frozen=True)
class ChunkPlacementPolicy:
    """Which chunks stay resident as always-visible windows (attention sinks + local context)."""

    keep_last: int = 1
    keep_first: int = 0
    first_token_level: bool = False

    def hot_first_range(self, n_closed: int) -> Tuple[int, int]:
        return 0, min(self.keep_first, n_closed)

    def hot_last_range(self, n_closed: int) -> Tuple[int, int]:
        if self.keep_last <= 0:
            return n_closed, n_closed
        lo = min(max(self.keep_first, n_closed - self.keep_last), n_closed)
        return lo, n_closed
