"""Multi-GPU prefill of one sequence: query chunks sharded across ranks, K/V and routing summaries
all-gathered once per layer.

The routed prefill of query chunk n reads only (a) chunk / group summaries of chunks < n and
(b) token K/V rows of its working set (windows, opened groups, its own chunk), so chunks are
independent once every rank holds the whole sequence's summaries and K/V
(ExistingModelFineTuning/KvRouter/vectorized.py:298-396 index only by query chunk).  Each rank:

  1. projects its own token rows (fused QKV GEMM) and runs the q/k RMSNorm + RoPE prologue, writing
     its K (RoPE'd) and V rows straight into its slice of a flat send buffer;
  2. builds the routing summaries of its own chunks into the same send buffer;
  3. one all-gather of the send buffers (K, V, chunk_k, group_k: group V summaries are not read by
     the token-only path) over NCCL, then one permuting copy per tensor into the [B, KVH, S, Dh]
     row layout the kernels address;
  4. routes and attends its own chunks (hga_route_prefill_range / hga_attend_prefill_range) and
     applies o_proj to its rows.

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
    """Element layout of one rank's send buffer: K rows, V rows, chunk_k, group_k (model dtype)."""
    B: int
    KVH: int
    Dh: int
    M: int
    rows: int          # token rows per rank (chunks per rank * C)
    chunks: int        # chunks per rank
    dtype: torch.dtype

    @property
    def elems(self) -> Tuple[int, int, int, int]:
        kv = self.B * self.KVH * self.rows * self.Dh
        ck = self.B * self.KVH * self.chunks * self.Dh
        return kv, kv, ck, ck * self.M

    @property
    def numel(self) -> int:
        return sum(self.elems)

    def views(self, flat: torch.Tensor):
        """(k_rope [B,KVH,rows,Dh], v, chunk_k [B,KVH,chunks,Dh], group_k [B,KVH,chunks,M,Dh]) views."""
        a, b, c, d = self.elems
        shapes = ((self.B, self.KVH, self.rows, self.Dh), (self.B, self.KVH, self.rows, self.Dh),
                  (self.B, self.KVH, self.chunks, self.Dh), (self.B, self.KVH, self.chunks, self.M, self.Dh))
        out, o = [], 0
        for n, shape in zip((a, b, c, d), shapes):
            out.append(flat[o:o + n].view(shape))
            o += n
        return tuple(out)


def unpack_gathered(lay: ShardLayout, recv: torch.Tensor, world: int, k_rope: torch.Tensor, v: torch.Tensor,
                    chunk_k: torch.Tensor, group_k: torch.Tensor) -> None:
    """Scatter the all-gathered buffers [world * numel] into whole-sequence tensors
    (k_rope / v [B,KVH,world*rows,Dh], chunk_k [B,KVH,world*chunks,Dh], group_k [...,M,Dh]):
    one permuting copy per tensor (rank r's rows land at r*rows)."""
    B, KVH, Dh, M = lay.B, lay.KVH, lay.Dh, lay.M
    stacked = recv.view(world, lay.numel)
    a, b, c, d = lay.elems
    offs = [0, a, a + b, a + b + c, a + b + c + d]
    shapes = [(lay.rows, Dh), (lay.rows, Dh), (lay.chunks, Dh), (lay.chunks, M * Dh)]
    for i, dst in enumerate((k_rope, v, chunk_k, group_k)):
        src = stacked[:, offs[i]:offs[i + 1]].view(world, B, KVH, *shapes[i])
        dst.view(B, KVH, world, *shapes[i]).copy_(src.permute(1, 2, 0, 3, 4))


class ShardedPrefill:
    """Sharded prefill of ``HierarchicalGlobalAttentionRouted`` layers over ``world`` ranks.

    ``exchange(send) -> recv`` performs the all-gather (default: ``torch.distributed`` on the
    default group: ``all_gather_into_tensor`` over NCCL); tests substitute an in-process exchange.
    Buffers are kept between calls of the same shape.
    """

    def __init__(self, world: int, rank: int, exchange: Optional[Callable[[torch.Tensor], torch.Tensor]] = None):
        self.world, self.rank = world, rank
        self.exchange = exchange if exchange is not None else self._dist_exchange
        self._bufs = {}

    def _dist_exchange(self, send: torch.Tensor) -> torch.Tensor:
        import torch.distributed as dist
        recv = self._buf("recv", (self.world * send.numel(),), send.dtype, send.device)
        if dist.get_backend() == "nccl":
            dist.all_gather_into_tensor(recv, send)
        else:
            dist.all_gather(list(recv.view(self.world, -1).unbind(0)), send)
        return recv

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
        kr_s, v_s, ck_s, gk_s = lay.views(send)
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

    def global_phase(self, m, state, recv: torch.Tensor) -> Optional[torch.Tensor]:
        """Steps 3-4: unpack the gathered K/V and summaries, route + attend own chunks, o_proj.
        Returns this rank's output rows [B, SQ, d_model] (None for a rank with no chunks)."""
        lay = state["lay"]
        dev = recv.device
        W = self.world
        rows, chunks = W * lay.rows, W * lay.chunks
        k_rope = self._buf("k_rope", (lay.B, lay.KVH, rows, lay.Dh), lay.dtype, dev)
        v = self._buf("v", (lay.B, lay.KVH, rows, lay.Dh), lay.dtype, dev)
        ck = self._buf("ck", (lay.B, lay.KVH, chunks, lay.Dh), lay.dtype, dev)
        gk = self._buf("gk", (lay.B, lay.KVH, chunks, lay.M, lay.Dh), lay.dtype, dev)
        unpack_gathered(lay, recv, W, k_rope, v, ck, gk)
        lo, hi = state["lo"], state["hi"]
        if hi <= lo:
            return None
        S, hp, q = state["S"], state["hp"], state["q"]
        routing = ops.route_prefill(hp, q, ck, gk, seq_len=S, chunk_range=(lo, hi))
        out_heads = ops.attend_prefill(hp, q, k_rope, v, routing["open_gid"], routing["open_t0"], seq_len=S,
                                       chunk_range=(lo, hi))            # [B,H,SQ,Dh] view of [B,SQ,H,Dh]
        B, SQ = q.shape[0], q.shape[2]
        return m.o_proj(out_heads.transpose(1, 2).reshape(B, SQ, m.nhead * m.head_dim))

    def forward(self, m, x_local: torch.Tensor, seq_len: int) -> Optional[torch.Tensor]:
        state, send = self.local_phase(m, x_local, seq_len)
        recv = self.exchange(send)
        return self.global_phase(m, state, recv)


__all__ = ["ShardedPrefill", "ShardLayout", "prefill_partition", "unpack_gathered"]
