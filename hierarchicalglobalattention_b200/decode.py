"""Incremental decode: ChunkRouter.decode_block (ExistingModelFineTuning/KvRouter/chunk_router.py:279-407)
on the device kernels (hga_append_tokens, hga_route_decode, hga_attend_decode, hga_summaries).

A block of L <= chunk_size new tokens per sequence is appended to the active chunk, routed against
the store's closed-chunk summaries, attended over the window / opened / active tokens, and - when
it completes the chunk - the chunk is closed into the store (summaries with fixed anchors and fp32
rotary rows, chunk_router.py:631-657).  The close runs after the block's attention is launched,
because the RAM tier's window slots are recycled by it.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch

from . import ops


@dataclass
class DecodeContext:
    """What a decode block's RoutedKV needs to run its attention (and the deferred chunk close)."""

    router: object
    layer: int
    params: object
    seq_pos: torch.Tensor
    routing: dict
    close_chunk: Optional[int]           # chunk index to close after the attention, or None
    close_rows: Optional[torch.Tensor] = None  # batch rows that close (mixed-length batches)
    done: bool = False

    def attend(self, q: torch.Tensor) -> torch.Tensor:
        store = self.router.store
        hot_k, hot_v = store.hot_buffers(self.layer)
        cold_k, cold_v = store.cold_buffers(self.layer)
        open_gid = self.routing["open_gid"]
        banked = store.bank_gather(self.layer, self.params, open_gid) if hasattr(store, "bank_gather") else None
        if banked is not None:
            # the RAM tier's VRAM bank: this step's opened groups were made resident (misses copied
            # from the pinned record); the attention reads them from HBM by bank slot
            cold_k, cold_v, open_gid = banked
        out = ops.attend_decode(self.params, q, self.seq_pos, hot_k, hot_v, store.hot_mode, cold_k, cold_v,
                                open_gid, self.routing["open_t0"])
        self.finish()
        return out

    def attend_dca(self, q_raw: torch.Tensor, dca_chunk: int, dca_ceil: int, theta: float) -> torch.Tensor:
        """Dual Chunk Attention of the block (qwen_routed_attention.py:247-283): q_raw [B,H,L,Dh]
        before RoPE; the store holds keys roped at their intra-chunk positions."""
        store = self.router.store
        hot_k, hot_v = store.hot_buffers(self.layer)
        cold_k, cold_v = store.cold_buffers(self.layer)
        open_gid = open_pos = self.routing["open_gid"]
        banked = store.bank_gather(self.layer, self.params, open_gid) if hasattr(store, "bank_gather") else None
        if banked is not None:
            cold_k, cold_v, open_gid = banked
        out = ops.attend_decode_dca(self.params, q_raw, self.seq_pos, hot_k, hot_v, store.hot_mode, cold_k, cold_v,
                                    open_gid, self.routing["open_t0"], dca_chunk, dca_ceil, theta, open_pos=open_pos)
        self.finish()
        return out

    def finish(self) -> None:
        if self.done:
            return
        self.done = True
        if self.close_chunk is not None:
            close_chunk(self.router, self.layer, self.params, self.close_chunk, rows=self.close_rows)
        if self.router._pending.get(self.layer) is self:
            self.router._pending.pop(self.layer, None)


def close_chunk(router, layer: int, hp, n, rows=None) -> None:
    """Summaries of the just-completed chunk(s) into the store (chunk_router.py:631-657).

    ``n`` is one chunk index for the whole batch, or (mixed lengths) a list of chunk indices for
    the batch rows ``rows``.
    """
    store = router.store
    C = router.cfg.chunk_size
    st = store.layer_buffers(layer)
    act = store.active_raw(layer)
    if rows is not None and len(rows) == act.shape[0] and len(set(n)) == 1 and list(rows) == list(range(len(rows))):
        rows, n = None, n[0]          # every row closes the same chunk: one batched launch
    if rows is None:
        k_act, v_act = store.active_rows(layer, n)
        cos, sin = router.chunk_rotary(n, act.device)
        store.ensure_capacity(layer, n + 1)
        st = store.layer_buffers(layer)
        ops.summaries(hp, act, k_act.contiguous(), v_act.contiguous(), cos, sin, seq_len=C, pos0=n * C,
                      rot_row0=n * C, out=(st.chunk_k, st.group_k, st.group_v), out_chunk0=n)
        store.on_chunk_closed(layer, n)
        store.mark_closed(layer, n + 1)
        return
    # per-sequence closes (different chunk indices): one batch-1 summary launch per closing row
    import copy
    hp1 = copy.copy(hp)
    hp1.batch = 1
    for b, nb in zip(rows, n):
        k_act, v_act = store.active_rows(layer, nb)
        cos, sin = router.chunk_rotary(nb, act.device)
        store.ensure_capacity(layer, nb + 1)
        st = store.layer_buffers(layer)
        ops.summaries(hp1, act[b:b + 1], k_act[b:b + 1].contiguous(), v_act[b:b + 1].contiguous(), cos, sin,
                      seq_len=C, pos0=nb * C, rot_row0=nb * C,
                      out=(st.chunk_k[b:b + 1], st.group_k[b:b + 1], st.group_v[b:b + 1]), out_chunk0=nb)
        store.on_chunk_closed(layer, nb, row=b)


def _pool_size(policy, n_closed: int) -> int:
    f_lo, f_hi = policy.hot_first_range(n_closed)
    l_lo, _ = policy.hot_last_range(n_closed)
    return max(0, l_lo - f_hi)


def decode_block(router, layer, q, k_rope, k_raw, v, start_pos):
    """Route + assemble one block of L new tokens inside the active chunk (uniform batch)."""
    from .router import RoutedKV
    prev = router._pending.get(layer)
    if prev is not None:
        prev.finish()
    cfg, store = router.cfg, router.store
    C = cfg.chunk_size
    B, H, L, Dh = q.shape
    n, c0 = start_pos // C, start_pos % C
    assert c0 + L <= C, "decode_block must stay within one chunk; feed chunk-by-chunk."
    n_closed = store.num_closed_chunks(layer)
    assert n_closed == n, f"active chunk {n} != closed {n_closed}; out-of-order block"
    hp = cfg.hga_params(store.policy, B, q.dtype)
    store.ensure_capacity(layer, max(n, 1), (n + 1) * C)
    seq_pos = router._seq_pos(B, start_pos, q.device)
    hot_k, hot_v = store.hot_buffers(layer)
    cold_k, cold_v = store.cold_buffers(layer)
    ops.append_tokens(hp, seq_pos, k_rope, v, k_raw, hot_k, hot_v, store.hot_mode,
                      None if store.hot_mode == 0 else cold_k, None if store.hot_mode == 0 else cold_v,
                      store.active_raw(layer))
    st = store.layer_buffers(layer)
    nmid = _pool_size(store.policy, n)
    if nmid > 0:
        routing = ops.route_decode(hp, q.contiguous(), seq_pos, st.chunk_k, st.group_k, nmid)
    else:
        z = torch.empty(B, H, 0, device=q.device, dtype=torch.int32)
        routing = {"mid_chunk": z, "mid_t0": z, "open_gid": z, "open_t0": z}
    router._active_len[layer] = (c0 + L) % C
    # chunk-summary lookups of this block (all HBM-resident: the summary bank spans the context)
    store.summary_hits += B * H * routing["mid_chunk"].shape[-1]
    ctx = DecodeContext(router, layer, hp, seq_pos, routing, n if c0 + L == C else None)
    router._pending[layer] = ctx
    return RoutedKV(params=hp, seq_len=L, token_k=hot_k, token_v=hot_v, routing=routing, scale=cfg.scale,
                    chunked=False, chunk_size=C, decode=ctx)


def decode_step(router, layer, q, k_rope, k_raw, v, seq_pos: torch.Tensor, seq_pos_host):
    """One block per sequence at per-sequence positions (mixed-length batches; no reference
    equivalent).  ``seq_pos`` device int32 [B], ``seq_pos_host`` the same as a Python list."""
    from .router import RoutedKV
    prev = router._pending.get(layer)
    if prev is not None:
        prev.finish()
    cfg, store = router.cfg, router.store
    C = cfg.chunk_size
    B, H, L, Dh = q.shape
    hp = cfg.hga_params(store.policy, B, q.dtype)
    nmax = max(seq_pos_host) // C
    store.ensure_capacity(layer, max(nmax, 1), (nmax + 1) * C)
    hot_k, hot_v = store.hot_buffers(layer)
    cold_k, cold_v = store.cold_buffers(layer)
    for pos in seq_pos_host:
        assert pos % C + L <= C, "decode_step blocks must stay within each sequence's chunk"
    ops.append_tokens(hp, seq_pos, k_rope, v, k_raw, hot_k, hot_v, store.hot_mode,
                      None if store.hot_mode == 0 else cold_k, None if store.hot_mode == 0 else cold_v,
                      store.active_raw(layer))
    st = store.layer_buffers(layer)
    nmid = max(_pool_size(store.policy, pos // C) for pos in seq_pos_host)
    if nmid > 0:
        routing = ops.route_decode(hp, q.contiguous(), seq_pos, st.chunk_k, st.group_k, nmid)
    else:
        z = torch.empty(B, H, 0, device=q.device, dtype=torch.int32)
        routing = {"mid_chunk": z, "mid_t0": z, "open_gid": z, "open_t0": z}
    store.summary_hits += B * H * routing["mid_chunk"].shape[-1]
    rows = [b for b, pos in enumerate(seq_pos_host) if pos % C + L == C]
    ctx = DecodeContext(router, layer, hp, seq_pos, routing, [seq_pos_host[b] // C for b in rows] if rows else None,
                        close_rows=rows if rows else None)
    router._pending[layer] = ctx
    return RoutedKV(params=hp, seq_len=L, token_k=hot_k, token_v=hot_v, routing=routing, scale=cfg.scale,
                    chunked=False, chunk_size=C, decode=ctx)
