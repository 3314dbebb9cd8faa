"""Multi-GPU prefill of one sequence: query chunks sharded across ranks, K/V and routing summaries
all-gathered once per layer.

The routed prefill of query chunk n reads only (a) chunk / group summaries of chunks < n and
(b) token K/V rows of its working set (windows, opened groups, its own chunk), so chunks are
independent once every rank holds the whole sequence's summaries and K/V
(ExistingModelFineTuning/KvRouter/vectorized.py:298-396 index only by query chunk).  Each rank:

  1. projects its own token rows (fused QKV GEMM) and runs the q/k RMSNorm + RoPE prologue, writing
     its K (RoPE'd) and V rows straight into its slice of a flat send buffer;
  2. builds the routing summaries of its own chunks into the same send buffer;
  3. all-gathers the routing summaries (chunk_k, group_k; group V summaries are not read by the
     token-only path) over NCCL and routes its own chunks (hga_route_prefill_range) while a second,
     asynchronous all-gather moves the K / V rows; each gathered tensor is put into the
     [B, KVH, S, Dh] row layout the kernels address by one permuting copy;
  4. attends its own chunks (hga_attend_prefill_range) and applies o_proj to its rows.

Partition: rank r owns chunks [r*P, min((r+1)*P, N)), P = ceil(N / world) — equal row counts, so
the all-gather needs no size exchange and the unpack is one strided copy per tensor.  The output
stays sharded (each rank returns its own rows).  The store is not seeded (decode after a sharded
prefill runs on one device per sequence).
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Callable, List, Optional, Tuple

import torch
import torch.nn.functional as F

from . import ops


def prefill_partition(seq_len: int, chunk_size: int, world: int) -> List[Tuple[int, int]]:
    """[(chunk_lo, chunk_hi)] per rank: equal chunk counts, the last ranks possibly short or empty."""
    N = (seq_len + chunk_size - 1) // chunk_size
    per = (N + world - 1) // world
    return [(min(r * per, N), min((r + 1) * per, N)) for r in range(world)]


@dataclass
class ShardLayout:
    """Element layout of one rank's send buffer: [chunk_k | group_k] (the routing part, gathered
    first) then [K rows | V rows] (the attention part, gathered while the router runs)."""
    B: int
    KVH: int
    Dh: int
    M: int
    rows: int          # token rows per rank (chunks per rank * C)
    chunks: int        # chunks per rank
    dtype: torch.dtype

    @property
    def sum_numel(self) -> int:
        return self.B * self.KVH * self.chunks * self.Dh * (1 + self.M)

    @property
    def kv_numel(self) -> int:
        return 2 * self.B * self.KVH * self.rows * self.Dh

    @property
    def numel(self) -> int:
        return self.sum_numel + self.kv_numel

    def views(self, flat: torch.Tensor):
        """(chunk_k [B,KVH,chunks,Dh], group_k [B,KVH,chunks,M,Dh], k_rope [B,KVH,rows,Dh], v) views."""
        ck = self.B * self.KVH * self.chunks * self.Dh
        kv = self.B * self.KVH * self.rows * self.Dh
        shapes = ((self.B, self.KVH, self.chunks, self.Dh), (self.B, self.KVH, self.chunks, self.M, self.Dh),
                  (self.B, self.KVH, self.rows, self.Dh), (self.B, self.KVH, self.rows, self.Dh))
        out, o = [], 0
        for n, shape in zip((ck, ck * self.M, kv, kv), shapes):
            out.append(flat[o:o + n].view(shape))
            o += n
        return tuple(out)


def _scatter(stacked: torch.Tensor, world: int, parts) -> None:
    """stacked [world, part elements...]: copy part i of every rank into dst_i (rank-major rows)."""
    o = 0
    for dst, n, shape in parts:
        src = stacked[:, o:o + n].view(world, *shape[:2], *shape[2:])
        B, KVH = shape[:2]
        dst.view(B, KVH, world, *shape[2:]).copy_(src.permute(1, 2, 0, 3, 4))
        o += n


def unpack_summaries(lay: ShardLayout, recv: torch.Tensor, world: int, chunk_k: torch.Tensor,
                     group_k: torch.Tensor) -> None:
    """Gathered routing parts [world * sum_numel] -> chunk_k [B,KVH,world*chunks,Dh] and group_k
    [B,KVH,world*chunks,M,Dh] (rank r's chunks land at r*chunks)."""
    ck = lay.B * lay.KVH * lay.chunks * lay.Dh
    _scatter(recv.view(world, lay.sum_numel), world,
             [(chunk_k, ck, (lay.B, lay.KVH, lay.chunks, lay.Dh)),
              (group_k, ck * lay.M, (lay.B, lay.KVH, lay.chunks, lay.M * lay.Dh))])


def unpack_kv(lay: ShardLayout, recv: torch.Tensor, world: int, k_rope: torch.Tensor, v: torch.Tensor) -> None:
    """Gathered attention parts [world * kv_numel] -> k_rope / v [B,KVH,world*rows,Dh]."""
    kv = lay.B * lay.KVH * lay.rows * lay.Dh
    shape = (lay.B, lay.KVH, lay.rows, lay.Dh)
    _scatter(recv.view(world, lay.kv_numel), world, [(k_rope, kv, shape), (v, kv, shape)])


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
        """Steps 1-2 for this rank: returns (state, send buffer).  x_local holds this rank's rows."""
        B = x_local.shape[0]
        KVH, Dh, C = m.kv_heads, m.head_dim, m.chunk_size
        M = C // m._cfg.group_size
        parts = prefill_partition(seq_len, C, self.world)
        per = parts[0][1] - parts[0][0]
        lo, hi = parts[self.rank]
        lay = ShardLayout(B, KVH, Dh, M, per * C, per, x_local.dtype)
        dev = x_local.device
        # zero-filled once: rows past the sequence end stay finite (the kernels stream whole units)
        send = self._buf("send", (lay.numel,), x_local.dtype, dev, zero=True)
        ck_s, gk_s, kr_s, v_s = lay.views(send)
        hp = m._cfg.hga_params(m._policy, B, x_local.dtype)
        state = {"lay": lay, "lo": lo, "hi": hi, "hp": hp, "S": seq_len}
        if hi <= lo:
            return state, send
        SQ = min(seq_len, hi * C) - lo * C
        if x_local.shape[1] != SQ:
            raise ValueError(f"rank {self.rank} owns rows [{lo * C}, {lo * C + SQ}); got {x_local.shape[1]} rows")
        w, b = m._fused_qkv()
        qkv = F.linear(x_local, w, b)
        cos, sin = m._own_rotary(seq_len, dev)
        qn = m.q_norm.weight.detach().to(x_local.dtype).contiguous() if hasattr(m.q_norm, "weight") else None
        kn = m.k_norm.weight.detach().to(x_local.dtype).contiguous() if hasattr(m.k_norm, "weight") else None
        kraw = self._buf("kraw", (B, KVH, per * C, Dh), x_local.dtype, dev)
        q, k_raw, k_rope, v = ops.qkv_prologue(hp, qkv, cos, sin, q_norm_w=qn, k_norm_w=kn, eps=m.norm_eps,
                                               norm_mode=0, rope_mode=0, rot_row0=0, pos0=lo * C,
                                               kv_out=(kraw, kr_s, v_s), kv_row0=0)
        ops.summaries(hp, k_raw, k_rope, v, cos, sin, seq_len=SQ, pos0=lo * C, rot_row0=0, round_table=True,
                      out=(ck_s, gk_s, None), out_chunk0=0, with_group_v=False)
        state["q"] = q
        return state, send

    def global_phase(self, m, state, recv_sum: torch.Tensor, recv_kv: torch.Tensor, kv_handle=None):
        """Steps 3-4: unpack the gathered summaries, route own chunks, (wait for the K/V gather)
        unpack K/V, attend, o_proj.  Returns this rank's output rows [B, SQ, d_model] (None for a
        rank with no chunks)."""
        lay = state["lay"]
        dev = recv_sum.device
        W = self.world
        rows, chunks = W * lay.rows, W * lay.chunks
        ck = self._buf("ck", (lay.B, lay.KVH, chunks, lay.Dh), lay.dtype, dev)
        gk = self._buf("gk", (lay.B, lay.KVH, chunks, lay.M, lay.Dh), lay.dtype, dev)
        unpack_summaries(lay, recv_sum, W, ck, gk)
        lo, hi = state["lo"], state["hi"]
        routing = None
        if hi > lo:
            routing = ops.route_prefill(state["hp"], state["q"], ck, gk, seq_len=state["S"], chunk_range=(lo, hi))
        if kv_handle is not None:
            kv_handle.wait()
        k_rope = self._buf("k_rope", (lay.B, lay.KVH, rows, lay.Dh), lay.dtype, dev)
        v = self._buf("v", (lay.B, lay.KVH, rows, lay.Dh), lay.dtype, dev)
        unpack_kv(lay, recv_kv, W, k_rope, v)
        if routing is None:
            return None
        q = state["q"]
        out_heads = ops.attend_prefill(state["hp"], q, k_rope, v, routing["open_gid"], routing["open_t0"],
                                       seq_len=state["S"], chunk_range=(lo, hi))   # [B,H,SQ,Dh] of [B,SQ,H,Dh]
        B, SQ = q.shape[0], q.shape[2]
        return m.o_proj(out_heads.transpose(1, 2).reshape(B, SQ, m.nhead * m.head_dim))

    def forward(self, m, x_local: torch.Tensor, seq_len: int) -> Optional[torch.Tensor]:
        state, send = self.local_phase(m, x_local, seq_len)
        lay = state["lay"]
        if self.exchange is not None:
            recv = self.exchange(send).view(self.world, lay.numel)
            return self.global_phase(m, state, recv[:, :lay.sum_numel].contiguous(),
                                     recv[:, lay.sum_numel:].contiguous())
        recv_sum, _ = self._gather("recv_sum", send[:lay.sum_numel], async_op=False)
        recv_kv, h = self._gather("recv_kv", send[lay.sum_numel:], async_op=True)
        return self.global_phase(m, state, recv_sum, recv_kv, h)


__all__ = ["ShardedPrefill", "ShardLayout", "prefill_partition", "unpack_summaries", "unpack_kv"]
