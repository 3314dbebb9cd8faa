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

VRAM token bank (``vram_cache_chunks`` > 0, the reference's bounded LRU bank,
ram_kv_cache_store.py:266-317): per layer and per (sequence, KV head) an HBM cache of 16-token
groups of the record with device-side slot maps.  Each decode step, ``hga_gather_h2d`` takes the
union of the groups a KV head's query heads opened, copies only the groups not in the bank (exact
LRU replacement) from the pinned record, and the attention reads the opened groups from the bank.
``vram_cache_chunks`` is an upper bound in chunks per layer (times groups_per_chunk slots per
sequence and KV head); like the reference the bank is sized down to the free device memory left
after ``vram_cache_reserve_gb`` (shared over ``num_layers``), and it is bypassed (groups read in
place from the pinned record) when it cannot hold one step's opened groups.  ``cache_hits`` /
``cache_misses`` count groups per (sequence, KV head) — the reference counts whole chunks per
batch.  Chunk and group summaries of every closed chunk are in HBM (the reference's summary bank
spanning the whole context): every summary lookup is a hit.

``pin_memory=False`` (the reference Qwen patch's default) is accepted: the decode kernels read the
record from device code, which needs page-locked memory, so the record is pinned regardless and a
warning says so.
"""
from __future__ import annotations

import warnings
from typing import Dict, Optional

import torch

from . import ops
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
        self.pin_memory = True
        if not pin_memory:
            warnings.warn("RamKVCacheStore(pin_memory=False): the B200 decode kernels read the cold record from "
                          "device code, so it is allocated in page-locked memory anyway", stacklevel=2)
        self.vram_cache_chunks = int(vram_cache_chunks)
        self.vram_summary_chunks = int(vram_summary_chunks)
        self.num_layers = int(num_layers)
        self.vram_cache_reserve_gb = float(vram_cache_reserve_gb)
        self.kf = max(0, int(policy.keep_first))
        self.kl = max(0, int(policy.keep_last))
        if self.kf + self.kl > 4096:
            raise ValueError("keep_first + keep_last windows larger than 4096 chunks belong in the VRAM tier")
        self._bank: Dict[int, dict] = {}
        self._bank_slots: Optional[int] = None            # resolved slots per (sequence, KV head)
        self._counters = torch.zeros(2, dtype=torch.int64, device=self.compute_device)   # hits, misses
        self._hits0 = self._misses0 = 0

    # -- counters (device-side for the bank, read on access) ------------------------------------
    @property
    def cache_hits(self) -> int:
        return self._hits0 + (int(self._counters[0].item()) if hasattr(self, "_counters") else 0)

    @cache_hits.setter
    def cache_hits(self, v: int) -> None:
        self._hits0 = int(v)
        if hasattr(self, "_counters"):
            self._counters[0].zero_()

    @property
    def cache_misses(self) -> int:
        return self._misses0 + (int(self._counters[1].item()) if hasattr(self, "_counters") else 0)

    @cache_misses.setter
    def cache_misses(self, v: int) -> None:
        self._misses0 = int(v)
        if hasattr(self, "_counters"):
            self._counters[1].zero_()

    # -- VRAM token bank --------------------------------------------------------------------------
    def _effective_slots(self) -> int:
        """Bank slots per (sequence, KV head): vram_cache_chunks * M, reduced to what the free device
        memory allows after vram_cache_reserve_gb, shared by num_layers layers (the reference's
        _effective_cap)."""
        if self._bank_slots is None:
            want = self.vram_cache_chunks * self.M
            if want > 0 and self.compute_device.type == "cuda":
                free, _ = torch.cuda.mem_get_info(self.compute_device)
                budget = free - self.vram_cache_reserve_gb * (1 << 30)
                per_slot = self.B * self.kvh * (self.C // self.M) * self.dh * 2 * self._elt() + self.B * self.kvh * 8
                fit = int(max(0, budget) // max(1, self.num_layers) // per_slot)
                want = min(want, fit)
            self._bank_slots = max(0, want)
        return self._bank_slots

    def _elt(self) -> int:
        return torch.empty((), dtype=self.dtype).element_size()

    def reset(self) -> None:
        self._bank.clear()
        super().reset()

    def bank_for(self, layer: int, need_slots: int) -> Optional[dict]:
        """The layer's bank (allocated on first use), or None when banking is off or the bank cannot
        hold ``need_slots`` groups per (sequence, KV head)."""
        slots = self._effective_slots()
        if slots <= 0 or slots < need_slots:
            return None
        st = self.layer_buffers(layer)
        gs = self.C // self.M
        gid_cap = st.tcap // gs
        bk = self._bank.get(layer)
        dev = self.compute_device
        if bk is None:
            bk = {"k": torch.zeros(self.B, self.kvh, slots * gs, self.dh, device=dev, dtype=self.dtype),
                  "v": torch.zeros(self.B, self.kvh, slots * gs, self.dh, device=dev, dtype=self.dtype),
                  "slot_gid": torch.full((self.B, self.kvh, slots), -1, dtype=torch.int32, device=dev),
                  "slot_stamp": torch.full((self.B, self.kvh, slots), -1, dtype=torch.int32, device=dev),
                  "gid_slot": torch.full((self.B, self.kvh, gid_cap), -1, dtype=torch.int32, device=dev),
                  "slots": slots, "stamp": 0}
            self._bank[layer] = bk
        elif bk["gid_slot"].shape[2] < gid_cap:
            # the record grew (capacity doubling): extend the gid -> slot map, keep the bank
            g = torch.full((self.B, self.kvh, gid_cap), -1, dtype=torch.int32, device=dev)
            g[:, :, :bk["gid_slot"].shape[2]] = bk["gid_slot"]
            bk["gid_slot"] = g
        return bk

    def bank_gather(self, layer: int, hp, open_gid: torch.Tensor):
        """One decode step's hga_gather_h2d: returns (bank_k, bank_v, open_slot) for the attention,
        or None (no bank: the attention reads the pinned record in place)."""
        H, Kg = open_gid.shape[1], open_gid.shape[2]
        bk = self.bank_for(layer, (H // self.kvh) * Kg)
        if bk is None or Kg == 0:
            return None
        st = self.layer_buffers(layer)
        open_slot = ops.gather_h2d(hp, open_gid, st.token_k, st.token_v, bk["k"], bk["v"], bk["slot_gid"],
                                   bk["gid_slot"], bk["slot_stamp"], bk["stamp"], self._counters)
        bk["stamp"] += 1
        return bk["k"], bk["v"], open_slot

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
