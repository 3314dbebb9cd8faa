"""Tiered KV-cache stores with device-native buffers.

Interface of the reference's ``KVCacheStore`` ABC (ExistingModelFineTuning/KvRouter/kv_cache_store.py:26-82)
plus ``seed_closed_chunks`` / ``gather_chunk_tokens_kvh`` and the hit/miss counters of
``RamKVCacheStore`` (ram_kv_cache_store.py:29-619), re-laid out for the B200 kernels:

* per layer, token K (RoPE applied) and V live in ``[B, KVH, cap, Dh]`` row buffers, so chunk ``i``
  is rows ``[i*C, (i+1)*C)`` of one contiguous (batch, kv-head) row block — the layout the
  attention kernels address directly (no per-chunk gathers, no head expansion);
* chunk summaries ``[B, KVH, ccap, Dh]`` and group summaries ``[B, KVH, ccap, M, Dh]`` stay in HBM
  for every closed chunk (180 GB per B200: a 131K-token layer's summaries are ~80 MB);
* ``VramKVCacheStore`` keeps token rows in HBM; ``RamKVCacheStore`` keeps the complete token record
  in pinned host memory (the cold tier) and the always-resident windows in HBM.

Capacities grow by doubling, as in the reference (ram_kv_cache_store.py:138-157).
"""
from __future__ import annotations

from abc import ABC, abstractmethod
from dataclasses import dataclass, field
from typing import Dict, Optional, Tuple

import torch

from .config import ChunkPlacementPolicy


class KVCacheStore(ABC):
    """Abstract tiered store; one instance serves all layers of a model."""

    def __init__(self, *, compute_device: torch.device, policy: ChunkPlacementPolicy) -> None:
        self.compute_device = torch.device(compute_device)
        self.policy = policy

    @abstractmethod
    def reset(self) -> None: ...

    @abstractmethod
    def num_closed_chunks(self, layer: int) -> int: ...

    @abstractmethod
    def chunk_summaries(self, layer: int) -> Optional[torch.Tensor]: ...

    @abstractmethod
    def append_closed_chunk(self, layer, chunk_k, group_k, group_v, token_k, token_v) -> None: ...

    @abstractmethod
    def gather_group_summaries(self, layer: int, chunk_idx: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]: ...

    @abstractmethod
    def gather_tokens(self, layer: int, chunk_idx: torch.Tensor, group_idx: torch.Tensor): ...

    @abstractmethod
    def hot_group_summaries(self, layer: int, lo: int, hi: int): ...

    @abstractmethod
    def hot_tokens(self, layer: int, lo: int, hi: int): ...

    def prefetch(self, layer: int, chunk_idx: torch.Tensor) -> None:  # noqa: B027 - optional hook
        """Best-effort hint; the device-resident tiers need none."""


@dataclass
class LayerBuffers:
    """Device-side (and, for the RAM tier, host-side) buffers of one layer."""

    n_closed: int = 0
    ccap: int = 0                                 # chunk capacity of the summary buffers
    tcap: int = 0                                 # token-row capacity of the token buffers
    chunk_k: Optional[torch.Tensor] = None        # [B,KVH,ccap,Dh]      device
    group_k: Optional[torch.Tensor] = None        # [B,KVH,ccap,M,Dh]    device
    group_v: Optional[torch.Tensor] = None        # [B,KVH,ccap,M,Dh]    device
    token_k: Optional[torch.Tensor] = None        # [B,KVH,tcap,Dh]      device (VRAM) / pinned host (RAM)
    token_v: Optional[torch.Tensor] = None
    active_raw: Optional[torch.Tensor] = None     # [B,KVH,C,Dh] pre-RoPE K of the active chunk (device)
    hot_k: Optional[torch.Tensor] = None          # RAM tier: [B,KVH,(kf+kl+1)*C,Dh] window/active slots (device)
    hot_v: Optional[torch.Tensor] = None


class VramKVCacheStore(KVCacheStore):
    """All-HBM tier (the reference's ``VramKVCacheStore``, vram_kv_cache_store.py:15-50)."""

    cold_on_host = False

    def __init__(self, *, compute_device, policy, kv_heads, head_dim, chunk_size, groups_per_chunk, batch_size,
                 dtype=torch.float32, initial_capacity: int = 64, **_unused) -> None:
        super().__init__(compute_device=compute_device, policy=policy)
        self.kvh, self.dh, self.C, self.M, self.B = kv_heads, head_dim, chunk_size, groups_per_chunk, batch_size
        self.dtype = dtype
        self._init_cap = int(initial_capacity)
        self._layers: Dict[int, LayerBuffers] = {}
        self.cache_hits = self.cache_misses = 0
        self.summary_hits = self.summary_misses = 0

    # -- buffers -----------------------------------------------------------------------------
    def layer_buffers(self, layer: int) -> LayerBuffers:
        st = self._layers.get(layer)
        if st is None:
            st = LayerBuffers()
            self._layers[layer] = st
        return st

    def _token_tensor(self, rows: int) -> torch.Tensor:
        # zero-filled: the tensor-core kernels stream whole 16-row units, so rows past the
        # valid length must hold finite values (a NaN in V would poison P.V even at P = 0)
        return torch.zeros(self.B, self.kvh, rows, self.dh, device=self.compute_device, dtype=self.dtype)

    def ensure_capacity(self, layer: int, n_chunks: int, n_tokens: Optional[int] = None) -> LayerBuffers:
        """Grow (by doubling) so that ``n_chunks`` closed chunks and ``n_tokens`` token rows fit."""
        st = self.layer_buffers(layer)
        n_tokens = n_chunks * self.C if n_tokens is None else n_tokens
        dev, dt = self.compute_device, self.dtype
        if n_chunks > st.ccap:
            cap = max(self._init_cap, 2 * st.ccap, n_chunks)
            ck = torch.zeros(self.B, self.kvh, cap, self.dh, device=dev, dtype=dt)
            gk = torch.zeros(self.B, self.kvh, cap, self.M, self.dh, device=dev, dtype=dt)
            gv = torch.zeros_like(gk)
            if st.chunk_k is not None:
                # whole old capacity: rows of a mixed-length batch may be ahead of n_closed
                n = st.ccap
                ck[:, :, :n] = st.chunk_k[:, :, :n]
                gk[:, :, :n] = st.group_k[:, :, :n]
                gv[:, :, :n] = st.group_v[:, :, :n]
            st.chunk_k, st.group_k, st.group_v, st.ccap = ck, gk, gv, cap
        if n_tokens > st.tcap:
            cap = max(self._init_cap * self.C, 2 * st.tcap, n_tokens)
            cap = (cap + self.C - 1) // self.C * self.C
            tk, tv = self._token_tensor(cap), self._token_tensor(cap)
            if st.token_k is not None and st.tcap:
                keep = min(st.tcap, cap)
                tk[:, :, :keep] = st.token_k[:, :, :keep]
                tv[:, :, :keep] = st.token_v[:, :, :keep]
            st.token_k, st.token_v, st.tcap = tk, tv, cap
        return st

    # -- decode-side views: hot rows (windows + active chunk), cold record, active pre-RoPE K ----
    hot_mode = 0  # hot rows are addressed like cold rows (one HBM record)

    def hot_buffers(self, layer: int):
        st = self.layer_buffers(layer)
        return st.token_k, st.token_v

    def cold_buffers(self, layer: int):
        st = self.layer_buffers(layer)
        return st.token_k, st.token_v

    def active_raw(self, layer: int) -> torch.Tensor:
        st = self.layer_buffers(layer)
        if st.active_raw is None:
            st.active_raw = torch.zeros(self.B, self.kvh, self.C, self.dh, device=self.compute_device, dtype=self.dtype)
        return st.active_raw

    def active_rows(self, layer: int, n: int):
        """Token K/V rows of (active) chunk n as [B,KVH,C,Dh] views."""
        st = self.layer_buffers(layer)
        sl = slice(n * self.C, (n + 1) * self.C)
        return st.token_k[:, :, sl], st.token_v[:, :, sl]

    def on_chunk_closed(self, layer: int, n: int, row: Optional[int] = None) -> None:
        """Hook after chunk n closed (the RAM tier moves it into its window slots)."""

    def after_seed(self, layer: int, seq_len: int, row: Optional[int] = None) -> None:
        """Hook after a prefill seeded tokens [0, seq_len) of every batch row, or of ``row`` (the
        RAM tier fills its hot slots)."""

    def adopt_tokens(self, layer: int, token_k: torch.Tensor, token_v: torch.Tensor) -> None:
        """Take ownership of freshly written [B,KVH,cap,Dh] token buffers (zero-copy prefill seed)."""
        st = self.layer_buffers(layer)
        st.token_k, st.token_v, st.tcap = token_k, token_v, token_k.shape[2]

    # -- KVCacheStore API -----------------------------------------------------------------------
    def reset(self) -> None:
        # the layers keep their buffers for the next sequence (no re-allocation, no zero fill: every
        # row already holds finite values, which is all the kernels need past the valid length)
        for st in self._layers.values():
            st.n_closed = 0
        self.cache_hits = self.cache_misses = 0
        self.summary_hits = self.summary_misses = 0

    def num_closed_chunks(self, layer: int) -> int:
        return self.layer_buffers(layer).n_closed

    def chunk_summaries(self, layer: int) -> Optional[torch.Tensor]:
        st = self.layer_buffers(layer)
        if st.chunk_k is None or st.n_closed == 0:
            return None
        return st.chunk_k[:, :, : st.n_closed]

    def append_closed_chunk(self, layer, chunk_k, group_k, group_v, token_k, token_v) -> None:
        st = self.layer_buffers(layer)
        i = st.n_closed
        st = self.ensure_capacity(layer, i + 1)
        st.chunk_k[:, :, i] = chunk_k
        st.group_k[:, :, i] = group_k
        st.group_v[:, :, i] = group_v
        self.write_tokens(layer, i * self.C, token_k, token_v)
        st.n_closed = i + 1

    def write_tokens(self, layer: int, row0: int, token_k: torch.Tensor, token_v: torch.Tensor) -> None:
        """Copy token rows [row0, row0+L) (inputs [B,KVH,L,Dh])."""
        st = self.layer_buffers(layer)
        L = token_k.shape[2]
        st.token_k[:, :, row0:row0 + L].copy_(token_k, non_blocking=True)
        st.token_v[:, :, row0:row0 + L].copy_(token_v, non_blocking=True)

    def seed_closed_chunks(self, layer, chunk_k, group_k, group_v, token_k, token_v) -> None:
        """Bulk ingest of N closed chunks (ram_kv_cache_store.py:483-526).  token_* [B,KVH,N,C,Dh]."""
        N = chunk_k.shape[2]
        st = self.ensure_capacity(layer, N)
        st.chunk_k[:, :, :N] = chunk_k
        st.group_k[:, :, :N] = group_k
        st.group_v[:, :, :N] = group_v
        B, KVH = token_k.shape[:2]
        self.write_tokens(layer, 0, token_k.reshape(B, KVH, N * self.C, self.dh),
                          token_v.reshape(B, KVH, N * self.C, self.dh))
        st.n_closed = N

    def mark_closed(self, layer: int, n_closed: int) -> None:
        self.layer_buffers(layer).n_closed = n_closed

    def _kvh_index(self, chunk_idx: torch.Tensor):
        B, H = chunk_idx.shape[:2]
        rep = H // self.kvh
        dev = self.compute_device
        b = torch.arange(B, device=dev).view(B, *([1] * (chunk_idx.ndim - 1)))
        kv = (torch.arange(H, device=dev) // rep).view(1, H, *([1] * (chunk_idx.ndim - 2)))
        return b, kv

    def gather_group_summaries(self, layer, chunk_idx):
        st = self.layer_buffers(layer)
        idx = chunk_idx.to(self.compute_device)
        b, kv = self._kvh_index(idx)
        return st.group_k[b, kv, idx], st.group_v[b, kv, idx]

    def gather_tokens(self, layer, chunk_idx, group_idx):
        st = self.layer_buffers(layer)
        gs = self.C // self.M
        cidx = chunk_idx.to(self.compute_device)
        tok = (cidx * self.C + group_idx.to(self.compute_device) * gs).unsqueeze(-1) + torch.arange(gs, device=cidx.device)
        b, kv = self._kvh_index(cidx)
        b, kv = b.unsqueeze(-1), kv.unsqueeze(-1)
        return st.token_k[b, kv, tok.to(st.token_k.device)].to(self.compute_device), \
            st.token_v[b, kv, tok.to(st.token_v.device)].to(self.compute_device)

    def gather_chunk_tokens_kvh(self, layer, chunk_idx):
        """Whole-chunk token K/V for chunk_idx [B,KVH,K] -> [B,KVH,K,C,Dh]."""
        st = self.layer_buffers(layer)
        B, KVH, K = chunk_idx.shape
        idx = chunk_idx.to(st.token_k.device)
        rows = (idx.unsqueeze(-1) * self.C + torch.arange(self.C, device=idx.device))
        b = torch.arange(B, device=idx.device).view(B, 1, 1, 1)
        g = torch.arange(KVH, device=idx.device).view(1, KVH, 1, 1)
        return st.token_k[b, g, rows].to(self.compute_device), st.token_v[b, g, rows].to(self.compute_device)

    def hot_tokens(self, layer, lo, hi):
        st = self.layer_buffers(layer)
        sl = slice(lo * self.C, hi * self.C)
        B = self.B
        k = st.token_k[:, :, sl].reshape(B, self.kvh, hi - lo, self.C, self.dh)
        v = st.token_v[:, :, sl].reshape(B, self.kvh, hi - lo, self.C, self.dh)
        return k.to(self.compute_device), v.to(self.compute_device)

    def hot_group_summaries(self, layer, lo, hi):
        st = self.layer_buffers(layer)
        return st.group_k[:, :, lo:hi], st.group_v[:, :, lo:hi]
