"""ChunkRouter / RoutedKV on the B200 kernels.

Same entry points, arguments and return contract as the reference's router
(ExistingModelFineTuning/KvRouter/chunk_router.py:93-516): ``route_query_block`` returns a list of
``(RoutedKV, lo, hi)`` segments and the caller runs ``routed.attend(q[:, :, lo:hi],
use_summaries=False)`` on each.  What changes is the representation: a ``RoutedKV`` holds the
*compact* working set (the selected chunk / group lists with their first-visible query row, plus
the store's token buffers) instead of materialised ``[B,H,N,R,Dh]`` K/V copies and
``[B,H,N,C,R]`` masks, and ``attend`` runs the working-set attention kernel over it.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Dict, List, Optional, Tuple

import torch

from . import _lib, ops
from .config import RouterConfig
from .store import KVCacheStore


@dataclass
class RoutedKV:
    """Compact routed context of one query block (data only; ``attend`` computes the attention).

    ``chunked`` (the chunk-parallel prefill): ``routing`` holds ``open_gid`` / ``open_t0``
    ``[B,H,N,Kg]`` and ``sel_chunk`` / ``sel_t0`` ``[B,H,N,Kc]``; keys are read from ``token_k`` /
    ``token_v`` ``[B,KVH,cap,Dh]`` rows [0, seq_len).
    """

    params: _lib.HgaParams
    seq_len: int
    token_k: torch.Tensor
    token_v: torch.Tensor
    routing: Dict[str, torch.Tensor]
    scale: float
    chunked: bool = False
    chunk_size: int = 0
    decode: Optional[object] = None
    out: Optional[torch.Tensor] = field(default=None, repr=False)  # optional [B,S,H,Dh] destination
    result: Optional[torch.Tensor] = field(default=None, repr=False)  # attention already computed

    def attend(self, q: torch.Tensor, use_summaries: bool = False) -> torch.Tensor:
        """Token-only attention over the routed keys: ``q`` [B,H,L,Dh] -> [B,H,L,Dh].

        Only the exact-token attention of the routed module is provided (the summary-attending
        variant is a different model family); ``use_summaries=True`` is rejected loudly.
        """
        if use_summaries:
            raise NotImplementedError("summary-attending attention is not part of the B200 hot path; "
                                      "call attend(q, use_summaries=False)")
        if self.result is not None:
            if self.result.shape != q.shape:
                raise ValueError("attend(q): q does not match the block this segment was routed for")
            return self.result
        if self.chunked:
            return ops.attend_prefill(self.params, q, self.token_k, self.token_v, self.routing["open_gid"],
                                      self.routing["open_t0"], seq_len=self.seq_len, out=self.out)
        return self.decode.attend(q)

    def attend_dca(self, q_raw: torch.Tensor, qpos: torch.Tensor, dca_chunk: int, dca_ceil: int,
                   theta: float) -> torch.Tensor:
        """Dual Chunk Attention over the routed keys (QwenRoutedAttention._dca_attend,
        qwen_routed_attention.py:247-283): ``q_raw`` [B,H,L,Dh] before RoPE, ``qpos`` the block's
        absolute positions (consecutive, from the segment's start).  Incremental segments only
        (route_query_block(..., return_positions=True))."""
        if self.decode is None:
            raise ValueError("attend_dca needs a segment routed with return_positions=True")
        return self.decode.attend_dca(q_raw, dca_chunk, dca_ceil, theta)


class ChunkRouter:
    """Router over a tiered store; chunk-parallel prefill and incremental decode."""

    def __init__(self, cfg: RouterConfig, store: KVCacheStore) -> None:
        self.cfg = cfg
        self.store = store
        self._active_len: Dict[int, int] = {}
        self._rot_cache: Dict[Tuple[str, int], Tuple[torch.Tensor, torch.Tensor]] = {}
        self._close_rot: Dict[Tuple[str, int], Tuple[torch.Tensor, torch.Tensor]] = {}
        self._pending: Dict[int, object] = {}   # decode blocks whose chunk close waits for their attention
        self._pos_cache: Dict[Tuple[int, int, str], torch.Tensor] = {}

    # ---------------------------------------------------------------------------------------
    def reset(self) -> None:
        for ctx in list(self._pending.values()):
            ctx.finish()
        self._pending.clear()
        self.store.reset()
        self._active_len.clear()

    def _seq_pos(self, B: int, pos: int, device) -> torch.Tensor:
        key = (B, pos, str(device))
        t = self._pos_cache.get(key)
        if t is None:
            if len(self._pos_cache) > 4096:
                self._pos_cache.clear()
            t = torch.full((B,), pos, dtype=torch.int32, device=device)
            self._pos_cache[key] = t
        return t

    def expected_position(self, layer: int) -> int:
        return self.store.num_closed_chunks(layer) * self.cfg.chunk_size + self._active_len.get(layer, 0)

    def is_empty(self, layer: int) -> bool:
        return self.expected_position(layer) == 0

    def rotary_table(self, start_pos: int, length: int, device) -> Tuple[torch.Tensor, torch.Tensor]:
        """fp32 cos/sin ``[1, 1, length, Dh]`` for positions [start_pos, start_pos+length)
        (chunk_router.py:457-461, 702-709)."""
        cos, sin = self._rotary(device, start_pos + length)
        e = start_pos + length
        return cos[start_pos:e].view(1, 1, length, -1), sin[start_pos:e].view(1, 1, length, -1)

    def _rotary(self, device, length: int) -> Tuple[torch.Tensor, torch.Tensor]:
        key = (str(device), 0)
        cached = self._rot_cache.get(key)
        if cached is None or cached[0].shape[0] < length:
            n = max(length, 2 * cached[0].shape[0] if cached is not None else length)
            # built with the host's fp32 cos/sin (the reference's own table) and uploaded once, so
            # closed-chunk summaries are bit-identical to the reference's
            half = self.cfg.head_dim // 2
            inv = 1.0 / (self.cfg.theta ** (torch.arange(half, dtype=torch.float32) / half))
            f = torch.arange(n, dtype=torch.float32).unsqueeze(-1) * inv
            emb = torch.cat((f, f), dim=-1)
            cached = (emb.cos().to(device), emb.sin().to(device))
            self._rot_cache[key] = cached
        return cached

    _ROT_RING = 16    # pinned staging slots for close tables

    def _rot_stage_ready(self) -> None:
        """Allocate the pinned staging ring of the close tables (1 MB at C=64, Dh=128) once, when a
        context is loaded for decode, rather than at the first chunk close of a decode loop."""
        if getattr(self, "_rot_stage", None) is None:
            C, Dh = self.cfg.chunk_size, self.cfg.head_dim
            self._rot_stage = torch.empty(self._ROT_RING, 2, C, Dh, dtype=torch.float32).pin_memory()
            self._rot_events = [None] * self._ROT_RING
            self._rot_slot = 0

    def chunk_rotary(self, n: int, device) -> Tuple[torch.Tensor, torch.Tensor]:
        """fp32 cos/sin ``[C, Dh]`` for the positions of chunk n (rows [n*C, n*C + C)), as the
        chunk-close summaries read them (their anchors, chunk_router.py:702-709).  Built on the host
        for a few KB per chunk and kept for the layers that close the same chunk.  The host table
        goes through a ring of pinned staging slots allocated once: a fresh pinned allocation
        per close could wait for the whole queued decode work, and a slot is reused only after
        the copy issued from it 16 closes earlier has completed."""
        key = (str(device), n)
        t = self._close_rot.get(key)
        if t is None:
            if len(self._close_rot) > 256:
                self._close_rot.clear()
            C, Dh = self.cfg.chunk_size, self.cfg.head_dim
            half = Dh // 2
            inv = 1.0 / (self.cfg.theta ** (torch.arange(half, dtype=torch.float32) / half))
            f = torch.arange(n * C, n * C + C, dtype=torch.float32).unsqueeze(-1) * inv
            emb = torch.cat((f, f), dim=-1)
            self._rot_stage_ready()
            slot = self._rot_slot
            self._rot_slot = (slot + 1) % self._ROT_RING
            if self._rot_events[slot] is not None:
                self._rot_events[slot].synchronize()
            stage = self._rot_stage[slot]
            torch.cos(emb, out=stage[0])
            torch.sin(emb, out=stage[1])
            dev_t = stage.to(device, non_blocking=True)
            ev = torch.cuda.Event()
            ev.record(torch.cuda.current_stream(device))
            self._rot_events[slot] = ev
            t = (dev_t[0], dev_t[1])
            self._close_rot[key] = t
        return t

    # ---------------------------------------------------------------------------------------
    def route_query_block(self, layer: int, q: torch.Tensor, k_rope: torch.Tensor, k_raw: torch.Tensor,
                          v: torch.Tensor, start_pos: int, cos: Optional[torch.Tensor] = None,
                          sin: Optional[torch.Tensor] = None, populate_store: bool = True,
                          max_chunks_at_once: Optional[int] = None, return_positions: bool = False,
                          _round_table: bool = False, _out: Optional[torch.Tensor] = None,
                          ) -> List[Tuple[RoutedKV, int, int]]:
        """Route a block of new queries (chunk_router.py:463-516).

        * the block stays inside one chunk -> one incremental ``decode_block`` segment;
        * a fresh multi-chunk block (start_pos 0) -> one chunk-parallel segment (summary builder,
          two-level router, working-set attention kernels), the store seeded from it;
        * multiple chunks over resident context -> one incremental segment per chunk.
        """
        C = self.cfg.chunk_size
        S = q.shape[2]
        first_chunk, last_chunk = start_pos // C, (start_pos + S - 1) // C
        if return_positions:
            # the Dual Chunk Attention caller: every block goes through the incremental path and
            # the caller attends each segment with RoutedKV.attend_dca, in order
            segs, p, done = [], start_pos, 0
            while done < S:
                take = min(C - (p % C), S - done)
                sl = slice(done, done + take)
                segs.append((self.decode_block(layer, q[:, :, sl], k_rope[:, :, sl], k_raw[:, :, sl], v[:, :, sl], p),
                             done, done + take))
                p += take
                done += take
            if len(segs) > 1 and self.store.hot_mode != 0:
                raise ValueError("return_positions over several chunks needs the VRAM tier (closing a chunk "
                                 "recycles the RAM tier's window slots before the caller attends); feed the "
                                 "block chunk by chunk")
            return segs
        if first_chunk == last_chunk:
            return [(self.decode_block(layer, q, k_rope, k_raw, v, start_pos), 0, S)]
        if start_pos == 0:
            return [(self._prefill_chunk_parallel(layer, q, k_rope, k_raw, v, cos, sin, populate_store,
                                                  _round_table, _out), 0, S)]
        # one incremental segment per chunk.  Each segment is attended before the next one is
        # routed: closing a chunk recycles store rows (the RAM tier's window and active slots) that
        # the previous segment's attention reads, so the attention cannot wait for the caller.
        segs = []
        p, done = start_pos, 0
        while done < S:
            take = min(C - (p % C), S - done)
            sl = slice(done, done + take)
            rk = self.decode_block(layer, q[:, :, sl], k_rope[:, :, sl], k_raw[:, :, sl], v[:, :, sl], p)
            rk.result = rk.attend(q[:, :, sl])
            segs.append((rk, done, done + take))
            p += take
            done += take
        return segs

    def _prefill_chunk_parallel(self, layer, q, k_rope, k_raw, v, cos, sin, populate_store, round_table, out):
        cfg, store = self.cfg, self.store
        B, H, S, Dh = q.shape
        C = cfg.chunk_size
        hp = cfg.hga_params(store.policy, B, q.dtype)
        if cos is None or sin is None:
            cos_t, sin_t = self._rotary(q.device, S)
            cos_t, sin_t = cos_t[:S], sin_t[:S]
            round_table = True
        else:
            cos_t, sin_t = cos.reshape(-1, Dh)[-S:], sin.reshape(-1, Dh)[-S:]
        n_closed = S // C
        if (populate_store and n_closed and cos_t.dtype == torch.float32 and ops.summaries_dual_supported(hp)):
            # (1) routing summaries and the store seed's closed-chunk summaries from one read of K/V
            self._rot_stage_ready()
            st = store.ensure_capacity(layer, max(n_closed, 1), S)
            cos32, sin32 = self._rotary(k_raw.device, S)
            ck, gk = ops.summaries_dual(hp, k_raw, k_rope, v, cos_t, sin_t, cos32, sin32,
                                        (st.chunk_k, st.group_k, st.group_v), n_closed, round_a=round_table)
            seeded = True
        else:
            # (1) routing summaries of the chunk-parallel path
            ck, gk, _ = ops.summaries(hp, k_raw, k_rope, v, cos_t, sin_t, round_table=round_table, with_group_v=False)
            seeded = False
        # (2) two-level routing
        routing = ops.route_prefill(hp, q, ck, gk)
        if populate_store:
            self._seed_store(layer, hp, k_rope, k_raw, v, S, summaries_done=seeded)
        return RoutedKV(params=hp, seq_len=S, token_k=k_rope, token_v=v, routing=routing, scale=cfg.scale,
                        chunked=True, chunk_size=C, out=out)

    def seed(self, layer: int, k_rope: torch.Tensor, k_raw: torch.Tensor, v: torch.Tensor) -> None:
        """Load a fresh context [0, S) into the store without attending over it (the store side of
        ``route_query_block(start_pos=0, populate_store=True)``); k_* / v [B,KVH,S,Dh]."""
        B = k_rope.shape[0]
        hp = self.cfg.hga_params(self.store.policy, B, k_rope.dtype)
        self._seed_store(layer, hp, k_rope, k_raw, v, k_rope.shape[2])

    def seed_mixed(self, layer: int, k_rope: torch.Tensor, k_raw: torch.Tensor, v: torch.Tensor,
                   seq_lens) -> None:
        """``seed`` for a batch whose sequences have different lengths (``seq_lens``, host ints):
        row b of k_* / v [B,KVH,Smax,Dh] holds its context in [0, seq_lens[b]).  Decode then
        continues through ``decode_step`` at per-sequence positions (no reference counterpart:
        the reference's batches share one position)."""
        import copy
        cfg, store = self.cfg, self.store
        C = cfg.chunk_size
        B = k_rope.shape[0]
        hp1 = copy.copy(cfg.hga_params(store.policy, B, k_rope.dtype))
        hp1.batch = 1
        self._rot_stage_ready()
        nmax = max(seq_lens) // C
        st = store.ensure_capacity(layer, max(nmax, 1), max(seq_lens) + C)
        store.write_tokens(layer, 0, k_rope, v)
        for b, S in enumerate(seq_lens):
            n = S // C
            if n:
                cos32, sin32 = self._rotary(k_raw.device, S)
                ops.summaries(hp1, k_raw[b:b + 1], k_rope[b:b + 1], v[b:b + 1], cos32, sin32, seq_len=n * C,
                              out=(st.chunk_k[b:b + 1], st.group_k[b:b + 1], st.group_v[b:b + 1]), out_chunk0=0)
            rem = S - n * C
            if rem:
                store.active_raw(layer)[b, :, :rem].copy_(k_raw[b, :, n * C:S])
            store.after_seed(layer, S, row=b)
        store.mark_closed(layer, min(seq_lens) // C)

    def _seed_store(self, layer, hp, k_rope, k_raw, v, S, summaries_done: bool = False):
        """Store seed of a fresh prefill (chunk_router.py:553-599): summaries of the closed chunks with
        fixed anchors and fp32 rotary rows (unless ``summaries_done``: written by hga_summaries_dual),
        token rows, and the partial active chunk."""
        self._rot_stage_ready()
        cfg, store = self.cfg, self.store
        C = cfg.chunk_size
        n_closed = S // C
        st = store.ensure_capacity(layer, max(n_closed, 1), S)
        if n_closed and not summaries_done:
            cos32, sin32 = self._rotary(k_raw.device, S)
            ops.summaries(hp, k_raw, k_rope, v, cos32, sin32, seq_len=n_closed * C,
                          out=(st.chunk_k, st.group_k, st.group_v), out_chunk0=0)
        if st.token_k.data_ptr() != k_rope.data_ptr():
            store.write_tokens(layer, 0, k_rope, v)
        store.mark_closed(layer, n_closed)
        rem = S - n_closed * C
        self._active_len[layer] = rem
        if rem:
            store.active_raw(layer)[:, :, :rem].copy_(k_raw[:, :, n_closed * C:])
        store.after_seed(layer, S)

    # ---------------------------------------------------------------------------------------
    def decode_block(self, layer, q, k_rope, k_raw, v, start_pos, return_positions: bool = False) -> RoutedKV:
        """Incremental routing of L <= chunk_size new tokens inside the active chunk
        (chunk_router.py:279-407).  q [B,H,L,Dh]; k_rope/k_raw/v [B,KVH,L,Dh]."""
        from .decode import decode_block
        return decode_block(self, layer, q, k_rope, k_raw, v, start_pos)

    def decode_step(self, layer, q, k_rope, k_raw, v, seq_pos: torch.Tensor, seq_pos_host) -> RoutedKV:
        """One block per sequence at per-sequence positions (mixed-length batched decode)."""
        from .decode import decode_step
        return decode_step(self, layer, q, k_rope, k_raw, v, seq_pos, seq_pos_host)

    def prefill(self, layer, q, k_rope, k_raw, v, start_pos: int = 0) -> torch.Tensor:
        """Stream a prefix chunk by chunk through the incremental path (chunk_router.py:410-442)."""
        C = self.cfg.chunk_size
        S = q.shape[2]
        outs, p, done = [], start_pos, 0
        while done < S:
            take = min(C - (p % C), S - done)
            sl = slice(done, done + take)
            routed = self.decode_block(layer, q[:, :, sl], k_rope[:, :, sl], k_raw[:, :, sl], v[:, :, sl], p)
            outs.append(routed.attend(q[:, :, sl], use_summaries=False))
            p += take
            done += take
        return torch.cat(outs, dim=2)
