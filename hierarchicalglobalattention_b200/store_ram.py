"""RAM tier: the complete token record in pinned host memory, windows and summaries in HBM.

Counterpart of the reference's ``RamKVCacheStore`` (ExistingModelFineTuning/KvRouter/ram_kv_cache_store.py:29-619).
Layout differences that the B200 kernels rely on:

* the cold record ``token_k/token_v [B, KVH, cap, Dh]`` is pinned host memory, reachable by the
  decode attention kernel through unified addressing: the opened groups' 4 KB rows are read over
  the host link inside the kernel (no staging copy, no Python LRU loop);
* a device slot buffer ``hot_k/hot_v [B, KVH, (kf + kl + 1) * C, Dh]`` holds the keep_first
  window (slot c), the keep_last window as a ring (slot kf + c % kl) and the active chunk
  (slot kf + kl): every window token is read from HBM;
* chunk and group summaries of every closed chunk stay in HBM (the reference's summary bank
  sized to span the whole context).

The reference's VRAM LRU token bank (``vram_cache_chunks``) and its hit/miss counters are kept as
attributes for interface compatibility; the zero-copy cold path does not use a bank.
"""
from __future__ import annotations

from typing import Optional

import torch

from .store import VramKVCacheStore


class RamKVCacheStore(VramKVCacheStore):
    """Pinned-host cold tier with HBM windows (see module docstring)."""

    cold_on_host = True
    hot_mode = 1

    def __init__(self, *, compute_device, policy, kv_heads, head_dim, chunk_size, groups_per_chunk, batch_size,
                 dtype=torch.float32, pin_memory: bool = True, initial_capacity: int = 64,
                 storage_device: Optional[torch.device] = None, vram_cache_chunks: int = 0,
                 vram_summary_chunks: int = 0, num_layers: int = 0, vram_cache_reserve_gb: float = 1.5,
                 **_unused) -> None:
        super().__init__(compute_device=compute_device, policy=policy, kv_heads=kv_heads, head_dim=head_dim,
                         chunk_size=chunk_size, groups_per_chunk=groups_per_chunk, batch_size=batch_size,
                         dtype=dtype, initial_capacity=initial_capacity)
        self.pin_memory = bool(pin_memory)
        if not self.pin_memory:
            raise ValueError("the B200 RAM tier reads the cold record from device code: pin_memory must be True")
        self.vram_cache_chunks = int(vram_cache_chunks)
        self.vram_summary_chunks = int(vram_summary_chunks)
        self.num_layers = int(num_layers)
        self.vram_cache_reserve_gb = float(vram_cache_reserve_gb)
        self.kf = max(0, int(policy.keep_first))
        self.kl = max(0, int(policy.keep_last))
        if self.kf + self.kl > 4096:
            raise ValueError("keep_first + keep_last windows larger than 4096 chunks belong in the VRAM tier")

    # -- buffers -----------------------------------------------------------------------------
    def _token_tensor(self, rows: int) -> torch.Tensor:
        return torch.zeros(self.B, self.kvh, rows, self.dh, dtype=self.dtype).pin_memory()

    def ensure_capacity(self, layer: int, n_chunks: int, n_tokens: Optional[int] = None):
        st = super().ensure_capacity(layer, n_chunks, n_tokens)
        if st.hot_k is None:
            rows = (self.kf + self.kl + 1) * self.C
            st.hot_k = torch.zeros(self.B, self.kvh, rows, self.dh, device=self.compute_device, dtype=self.dtype)
            st.hot_v = torch.zeros_like(st.hot_k)
        return st

    def hot_buffers(self, layer: int):
        st = self.layer_buffers(layer)
        return st.hot_k, st.hot_v

    def _slot(self, c: int) -> int:
        return c if c < self.kf else self.kf + (c % self.kl if self.kl > 0 else 0)

    def active_rows(self, layer: int, n: int):
        st = self.layer_buffers(layer)
        s = (self.kf + self.kl) * self.C
        return st.hot_k[:, :, s:s + self.C], st.hot_v[:, :, s:s + self.C]

    def write_tokens(self, layer: int, row0: int, token_k: torch.Tensor, token_v: torch.Tensor) -> None:
        st = self.layer_buffers(layer)
        L = token_k.shape[2]
        st.token_k[:, :, row0:row0 + L].copy_(token_k)
        st.token_v[:, :, row0:row0 + L].copy_(token_v)

    def _to_slot(self, layer: int, c: int, src_k: torch.Tensor, src_v: torch.Tensor, row: Optional[int],
                 dst_row: Optional[int] = None) -> None:
        """Copy chunk c's rows (batch row ``row`` of src, all rows if None) into its window slots
        (batch row ``dst_row``, default the same as ``row``)."""
        st = self.layer_buffers(layer)
        dst_row = row if dst_row is None else dst_row
        bs = slice(None) if row is None else slice(row, row + 1)
        bd = slice(None) if dst_row is None else slice(dst_row, dst_row + 1)
        dsts = []
        if c < self.kf:
            dsts.append(c)
        if self.kl > 0:
            dsts.append(self.kf + c % self.kl)
        for slot in dsts:
            sl = slice(slot * self.C, (slot + 1) * self.C)
            st.hot_k[bd, :, sl].copy_(src_k[bs], non_blocking=True)
            st.hot_v[bd, :, sl].copy_(src_v[bs], non_blocking=True)

    def on_chunk_closed(self, layer: int, n: int, row: Optional[int] = None) -> None:
        """The closed active chunk enters the keep_last ring (and the keep_first window)."""
        k_act, v_act = self.active_rows(layer, n)
        self._to_slot(layer, n, k_act.clone(), v_act.clone(), row)

    def after_seed(self, layer: int, seq_len: int, row: Optional[int] = None) -> None:
        """Fill the window / active slots after a prefill wrote the record (ram_kv_cache_store.py:511-526),
        for every batch row or only ``row``."""
        st = self.layer_buffers(layer)
        C = self.C
        n = seq_len // C
        f_lo, f_hi = self.policy.hot_first_range(n)
        l_lo, l_hi = self.policy.hot_last_range(n)
        bs = slice(None) if row is None else slice(row, row + 1)
        for c in sorted(set(range(f_lo, f_hi)) | set(range(l_lo, l_hi))):
            sl = slice(c * C, (c + 1) * C)
            self._to_slot(layer, c, st.token_k[bs, :, sl].to(self.compute_device),
                          st.token_v[bs, :, sl].to(self.compute_device), None if row is None else 0, row)
        rem = seq_len - n * C
        if rem:
            k_act, v_act = self.active_rows(layer, n)
            k_act[bs, :, :rem].copy_(st.token_k[bs, :, n * C:seq_len])
            v_act[bs, :, :rem].copy_(st.token_v[bs, :, n * C:seq_len])

    def hot_tokens(self, layer, lo, hi):
        st = self.layer_buffers(layer)
        sl = slice(lo * self.C, hi * self.C)
        k = st.token_k[:, :, sl].reshape(self.B, self.kvh, hi - lo, self.C, self.dh)
        v = st.token_v[:, :, sl].reshape(self.B, self.kvh, hi - lo, self.C, self.dh)
        return k.to(self.compute_device), v.to(self.compute_device)
