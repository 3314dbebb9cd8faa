"""Multi-GPU prefill of one sequence: query chunks sharded across ranks, K/V and routing summaries
all-gathered once per layer.

The routed prefill of query chunk n reads only (a) chunk / group summaries of chunks < n and
(b) token K/V rows of its working set (windows, opened groups, its own chunk), so chunks are
independent once every rank holds the whole sequence's summaries and K/V
(ExistingModelFineTuning/KvRouter/vectorized.py:298-396 index only by query chunk).  Each rank:

  1. projects its own token rows (fused QKV GEMM) and runs the q/k RMSNorm + RoPE prologue, writing
     its K (RoPE'd) and V rows straight into a flat send buffer;
  2. builds the routing summaries of its own chunks into the same send buffer;
  3. all-gathers the routing summaries (chunk_k, group_k; group V summaries are not read by the
     token-only path) over NCCL and routes its own chunks (hga_route_prefill_range) while a second,
     asynchronous all-gather moves the K / V rows; hga_shard_unpack puts each gathered part into
     the [B, KVH, S, Dh] row layout the kernels address;
  4. attends its own chunks (hga_attend_prefill_range) and applies o_proj to its rows.

Partition ("zigzag"): the chunks are cut into 2*world equal blocks and rank r owns blocks r and
2*world-1-r.  The router's work per chunk grows with the chunk index (its pool is every earlier
chunk), so pairing an early block with a late one gives every rank the same work; equal block
sizes keep the all-gather free of a size exchange.  The output stays sharded (each rank returns
the rows of its two blocks, in order).  The store is not seeded (decode after a sharded prefill
runs on one device per sequence).
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Callable, List, Optional, Tuple

import torch
import torch.nn.functional as F

from . import ops

PIECES = 2


def prefill_partition(seq_len: int, chunk_size: int, world: int) -> List[List[Tuple[int, int]]]:
    """Per rank, its two (chunk_lo, chunk_hi) blocks: blocks r and 2*world-1-r of 2*world equal
    blocks of ceil(N / (2*world)) chunks (late blocks may be short or empty)."""
    N = (seq_len + chunk_size - 1) // chunk_size
    P = (N + PIECES * world - 1) // (PIECES * world)
    blk = lambda i: (min(i * P, N), min((i + 1) * P, N))  # noqa: E731
    return [[blk(r), blk(PIECES * world - 1 - r)] for r in range(world)]


def block_table(world: int) -> List[int]:
    """Sequence block of piece j of rank r, flattened [r * PIECES + j]."""
    return [b for r in range(world) for b in (r, PIECES * world - 1 - r)]


def rank_rows(seq_len: int, chunk_size: int, world: int, rank: int) -> List[Tuple[int, int]]:
    """The token row ranges [(lo, hi)] of a rank's blocks (its input / output rows, in order)."""
    return [(lo * chunk_size, min(seq_len, hi * chunk_size)) for lo, hi in
            prefill_partition(seq_len, chunk_size, world)[rank] if hi > lo]


@dataclass
class ShardLayout:
    """Element layout of one rank's send buffer: [chunk_k | group_k] (the routing part, gathered
    first) then [K | V] (the attention part, gathered while the router runs); each tensor holds
    PIECES blocks of [B, KVH, chunks (or rows), ...]."""
    B: int
    KVH: int
    Dh: int
    M: int
    rows: int          # token rows per block (chunks per block * C)
    chunks: int        # chunks per block
    dtype: torch.dtype

    @property
    def ck_numel(self) -> int:
        return PIECES * self.B * self.KVH * self.chunks * self.Dh

    @property
    def k_numel(self) -> int:
        return PIECES * self.B * self.KVH * self.rows * self.Dh

    @property
    def sum_numel(self) -> int:
        return self.ck_numel * (1 + self.M)

    @property
    def kv_numel(self) -> int:
        return 2 * self.k_numel

    @property
    def numel(self) -> int:
        return self.sum_numel + self.kv_numel

    def views(self, flat: torch.Tensor):
        """(chunk_k [P,B,KVH,chunks,Dh], group_k [P,B,KVH,chunks,M,Dh], k_rope [P,B,KVH,rows,Dh], v)."""
        P, B, KVH, Dh = PIECES, self.B, self.KVH, self.Dh
        parts = ((self.ck_numel, (P, B, KVH, self.chunks, Dh)), (self.ck_numel * self.M, (P, B, KVH, self.chunks, self.M, Dh)),
                 (self.k_numel, (P, B, KVH, self.rows, Dh)), (self.k_numel, (P, B, KVH, self.rows, Dh)))
        out, o = [], 0
        for n, shape in parts:
            out.append(flat[o:o + n].view(shape))
            o += n
        return tuple(out)


class ShardedPrefill:
    """Sharded prefill of ``HierarchicalGlobalAttentionRouted`` layers over ``world`` ranks.

    ``exchange(send) -> recv`` replaces the collective (tests emulate the ranks in one process);
    by default the routing parts are all-gathered first and the K/V parts are all-gathered
    asynchronously over NCCL while the router runs.  Buffers are kept between calls of the same
    shape.
    """

    def __init__(self, world: int, rank: int, exchange: Optional[Callable[[torch.Tensor], torch.Tensor]] = None):
        self.world, self.rank = world, rank
        self.exchange = exchange
        self._bufs = {}

    def _gather(self, name, send: torch.Tensor, async_op: bool):
        import torch.distributed as dist
        recv = self._buf(name, (self.world * send.numel(),), send.dtype, send.device)
        if dist.get_backend() == "nccl":
            h = dist.all_gather_into_tensor(recv, send, async_op=async_op)
        else:
            h = dist.all_gather(list(recv.view(self.world, -1).unbind(0)), send, async_op=async_op)
        return recv, h

    def _buf(self, name, shape, dtype, device, zero=False):
        key = (name, tuple(shape), dtype, str(device))
        t = self._bufs.get(key)
        if t is None:
            t = (torch.zeros if zero else torch.empty)(shape, dtype=dtype, device=device)
            self._bufs[key] = t
        return t

    # ------------------------------------------------------------------------------------------
    def local_phase(self, m, x_local: torch.Tensor, seq_len: int):
        """Steps 1-2 for this rank: returns (state, send buffer).  x_local holds this rank's rows
        (``rank_rows``), its blocks one after the other."""
        B = x_local.shape[0]
        KVH, Dh, C = m.kv_heads, m.head_dim, m.chunk_size
        M = C // m._cfg.group_size
        blocks = prefill_partition(seq_len, C, self.world)[self.rank]
        per = prefill_partition(seq_len, C, self.world)[0][0][1]  # chunks per block
        lay = ShardLayout(B, KVH, Dh, M, per * C, per, x_local.dtype)
        dev = x_local.device
        # zero-filled once: rows past the sequence end stay finite (the kernels stream whole units)
        send = self._buf("send", (lay.numel,), x_local.dtype, dev, zero=True)
        ck_s, gk_s, kr_s, v_s = lay.views(send)
        hp = m._cfg.hga_params(m._policy, B, x_local.dtype)
        rows = sum(min(seq_len, hi * C) - lo * C for lo, hi in blocks if hi > lo)
        if x_local.shape[1] != rows:
            raise ValueError(f"rank {self.rank} owns {rows} rows ({blocks}); got {x_local.shape[1]}")
        state = {"lay": lay, "blocks": blocks, "hp": hp, "S": seq_len, "q": []}
        if rows == 0:
            return state, send
        w, b = m._fused_qkv()
        qkv = F.linear(x_local, w, b)
        cos, sin = m._own_rotary(seq_len, dev)
        qn = m.q_norm.weight.detach().to(x_local.dtype).contiguous() if hasattr(m.q_norm, "weight") else None
        kn = m.k_norm.weight.detach().to(x_local.dtype).contiguous() if hasattr(m.k_norm, "weight") else None
        kraw = self._buf("kraw", (B, KVH, per * C, Dh), x_local.dtype, dev)
        r0 = 0
        for j, (lo, hi) in enumerate(blocks):
            if hi <= lo:
                state["q"].append(None)
                continue
            SQ = min(seq_len, hi * C) - lo * C
            q, k_raw, k_rope, v = ops.qkv_prologue(hp, qkv[:, r0:r0 + SQ], cos, sin, q_norm_w=qn, k_norm_w=kn,
                                                   eps=m.norm_eps, norm_mode=0, rope_mode=0, rot_row0=0,
                                                   pos0=lo * C, kv_out=(kraw, kr_s[j], v_s[j]), kv_row0=0)
            ops.summaries(hp, k_raw, k_rope, v, cos, sin, seq_len=SQ, pos0=lo * C, rot_row0=0, round_table=True,
                          out=(ck_s[j], gk_s[j], None), out_chunk0=0, with_group_v=False)
            state["q"].append(q)
            r0 += SQ
        return state, send

    def _unpack(self, lay: ShardLayout, recv: torch.Tensor, rank_elems: int, offset_elems: int, rows: int,
                row_elems: int, dst: torch.Tensor) -> None:
        es = recv.element_size()
        ops.shard_unpack(recv, rank_elems * es, offset_elems * es, self.world, PIECES, block_table(self.world),
                         lay.B * lay.KVH, rows, row_elems * es, dst)

    def global_phase(self, m, state, recv_sum: torch.Tensor, recv_kv: torch.Tensor, kv_handle=None):
        """Steps 3-4: unpack the gathered summaries, route own chunks, (wait for the K/V gather)
        unpack K/V, attend, o_proj.  Returns this rank's output rows [B, rows, d_model] (None for a
        rank with no chunks)."""
        lay = state["lay"]
        dev = recv_sum.device
        W = self.world
        nblk = PIECES * W
        ck = self._buf("ck", (lay.B, lay.KVH, nblk * lay.chunks, lay.Dh), lay.dtype, dev)
        gk = self._buf("gk", (lay.B, lay.KVH, nblk * lay.chunks, lay.M, lay.Dh), lay.dtype, dev)
        self._unpack(lay, recv_sum, lay.sum_numel, 0, lay.chunks, lay.Dh, ck)
        self._unpack(lay, recv_sum, lay.sum_numel, lay.ck_numel, lay.chunks, lay.M * lay.Dh, gk)
        S, hp = state["S"], state["hp"]
        routings = []
        for (lo, hi), q in zip(state["blocks"], state["q"]):
            routings.append(ops.route_prefill(hp, q, ck, gk, seq_len=S, chunk_range=(lo, hi)) if q is not None
                            else None)
        if kv_handle is not None:
            kv_handle.wait()
        k_rope = self._buf("k_rope", (lay.B, lay.KVH, nblk * lay.rows, lay.Dh), lay.dtype, dev)
        v = self._buf("v", (lay.B, lay.KVH, nblk * lay.rows, lay.Dh), lay.dtype, dev)
        self._unpack(lay, recv_kv, lay.kv_numel, 0, lay.rows, lay.Dh, k_rope)
        self._unpack(lay, recv_kv, lay.kv_numel, lay.k_numel, lay.rows, lay.Dh, v)
        live = [(lo, hi, q, r) for (lo, hi), q, r in zip(state["blocks"], state["q"], routings) if q is not None]
        if not live:
            return None
        C = m.chunk_size
        sqs = [min(S, hi * C) - lo * C for lo, hi, _, _ in live]
        if lay.B == 1 and len(live) > 1:
            # one sequence: each block's rows are a contiguous slice of the rank's [1, rows, H, Dh]
            # output, which the attention writes in place (no concatenation copy)
            heads = self._buf("heads", (1, sum(sqs), m.nhead, m.head_dim), lay.dtype, dev)
            r0 = 0
            for (lo, hi, q, routing), sq in zip(live, sqs):
                ops.attend_prefill(hp, q, k_rope, v, routing["open_gid"], routing["open_t0"], seq_len=S,
                                   chunk_range=(lo, hi), out=heads[:, r0:r0 + sq])
                r0 += sq
        else:
            outs = [ops.attend_prefill(hp, q, k_rope, v, routing["open_gid"], routing["open_t0"], seq_len=S,
                                       chunk_range=(lo, hi)).transpose(1, 2)   # [B,SQ,H,Dh]
                    for lo, hi, q, routing in live]
            heads = outs[0] if len(outs) == 1 else torch.cat(outs, dim=1)
        B, R = heads.shape[:2]
        return m.o_proj(heads.reshape(B, R, m.nhead * m.head_dim))

    def forward(self, m, x_local: torch.Tensor, seq_len: int) -> Optional[torch.Tensor]:
        state, send = self.local_phase(m, x_local, seq_len)
        lay = state["lay"]
        if self.exchange is not None:
            recv = self.exchange(send).view(self.world, lay.numel)
            return self.global_phase(m, state, recv[:, :lay.sum_numel].contiguous().view(-1),
                                     recv[:, lay.sum_numel:].contiguous().view(-1))
        recv_sum, _ = self._gather("recv_sum", send[:lay.sum_numel], async_op=False)
        recv_kv, h = self._gather("recv_kv", send[lay.sum_numel:], async_op=True)
        return self.global_phase(m, state, recv_sum, recv_kv, h)


__all__ = ["ShardedPrefill", "ShardLayout", "prefill_partition", "block_table", "rank_rows", "PIECES"]
