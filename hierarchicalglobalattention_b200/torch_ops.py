"""The C ABI's entry points as PyTorch dispatcher operators, ``torch.ops.hga.*``.

Registered with ``torch.library`` (schema, CUDA implementation through ``ops``, and a fake /
meta implementation giving output shapes, so the operators trace under FakeTensorMode and
torch.compile without running).  The layer parameters travel as two lists (schemas take no
structs): ``pi`` = [batch, nhead, kv_heads, head_dim, chunk_size, group_size, topk_chunks,
topk_groups, keep_first, keep_last, cutoff_pair, dtype code] and ``pf`` = [scale,
group_kv_scale]; ``params_lists(p)`` builds them from an ``HgaParams``.

Operators (the C entry point each wraps):
  hga::summaries      (hga_summaries)        -> chunk_k, group_k, group_v
  hga::route_prefill  (hga_route_prefill)    -> sel_chunk, sel_t0, open_gid, open_t0
  hga::attend_prefill (hga_attend_prefill)   -> out [B,S,H,Dh]
  hga::route_decode   (hga_route_decode)     -> mid_chunk, mid_t0, open_gid, open_t0
  hga::attend_decode  (hga_attend_decode)    -> out [B,H,L,Dh]
  hga::attend_decode_dca (hga_attend_decode_dca) -> out [B,H,L,Dh]
  hga::gather_h2d     (hga_gather_h2d)       -> open_slot (mutates the bank and its maps)
"""
from __future__ import annotations

from typing import List, Optional, Tuple

import torch
from torch import Tensor

from . import _lib, ops


def params_lists(p: _lib.HgaParams) -> Tuple[List[int], List[float]]:
    return ([p.batch, p.nhead, p.kv_heads, p.head_dim, p.chunk_size, p.group_size, p.topk_chunks, p.topk_groups,
             p.keep_first, p.keep_last, p.cutoff_pair, p.dtype], [float(p.scale), float(p.group_kv_scale)])


def _params(pi: List[int], pf: List[float]) -> _lib.HgaParams:
    names = ["batch", "nhead", "kv_heads", "head_dim", "chunk_size", "group_size", "topk_chunks", "topk_groups",
             "keep_first", "keep_last", "cutoff_pair", "dtype"]
    if len(pi) != len(names) or len(pf) != 2:
        raise _lib.HgaError("hga ops: pi needs 12 ints and pf 2 floats (see params_lists)")
    return _lib.HgaParams(**dict(zip(names, (int(x) for x in pi))), scale=pf[0], group_kv_scale=pf[1])


# ---- summaries ------------------------------------------------------------------------------
@torch.library.custom_op("hga::summaries", mutates_args=())
def summaries(pi: List[int], pf: List[float], k_raw: Tensor, k_rope: Tensor, v: Tensor, cos: Tensor, sin: Tensor,
              round_table: bool) -> Tuple[Tensor, Tensor, Tensor]:
    ck, gk, gv = ops.summaries(_params(pi, pf), k_raw, k_rope, v, cos, sin, round_table=round_table)
    return ck, gk, gv


@summaries.register_fake
def _(pi, pf, k_raw, k_rope, v, cos, sin, round_table):
    B, KVH, S, Dh = k_raw.shape
    C, gs = pi[4], pi[5]
    N, M = (S + C - 1) // C, C // gs
    return (k_raw.new_empty(B, KVH, N, Dh), k_raw.new_empty(B, KVH, N, M, Dh), k_raw.new_empty(B, KVH, N, M, Dh))


# ---- prefill routing and attention ----------------------------------------------------------
@torch.library.custom_op("hga::route_prefill", mutates_args=())
def route_prefill(pi: List[int], pf: List[float], q: Tensor, chunk_k: Tensor, group_k: Tensor
                  ) -> Tuple[Tensor, Tensor, Tensor, Tensor]:
    r = ops.route_prefill(_params(pi, pf), q, chunk_k, group_k)
    return r["sel_chunk"], r["sel_t0"], r["open_gid"], r["open_t0"]


@route_prefill.register_fake
def _(pi, pf, q, chunk_k, group_k):
    B, H, S, _ = q.shape
    N, Kc, Kg, _ = ops.route_sizes(_params(pi, pf), S)
    i32 = dict(dtype=torch.int32, device=q.device)
    return (torch.empty(B, H, N, Kc, **i32), torch.empty(B, H, N, Kc, **i32), torch.empty(B, H, N, Kg, **i32),
            torch.empty(B, H, N, Kg, **i32))


@torch.library.custom_op("hga::attend_prefill", mutates_args=())
def attend_prefill(pi: List[int], pf: List[float], q: Tensor, k_rope: Tensor, v: Tensor, open_gid: Tensor,
                   open_t0: Tensor) -> Tensor:
    out = ops.attend_prefill(_params(pi, pf), q, k_rope, v, open_gid, open_t0, out_layout=ops.Q_BSHD)
    return out.transpose(1, 2)  # the [B,S,H,Dh] buffer itself


@attend_prefill.register_fake
def _(pi, pf, q, k_rope, v, open_gid, open_t0):
    B, H, S, Dh = q.shape
    return q.new_empty(B, S, H, Dh)


# ---- decode ---------------------------------------------------------------------------------
@torch.library.custom_op("hga::route_decode", mutates_args=())
def route_decode(pi: List[int], pf: List[float], q: Tensor, seq_pos: Tensor, chunk_k: Tensor, group_k: Tensor,
                 nmid_max: int) -> Tuple[Tensor, Tensor, Tensor, Tensor]:
    r = ops.route_decode(_params(pi, pf), q, seq_pos, chunk_k, group_k, nmid_max)
    return r["mid_chunk"], r["mid_t0"], r["open_gid"], r["open_t0"]


@route_decode.register_fake
def _(pi, pf, q, seq_pos, chunk_k, group_k, nmid_max):
    B, H = q.shape[:2]
    Kc, Kg = ops.decode_sizes(_params(pi, pf), nmid_max)
    i32 = dict(dtype=torch.int32, device=q.device)
    return (torch.empty(B, H, Kc, **i32), torch.empty(B, H, Kc, **i32), torch.empty(B, H, Kg, **i32),
            torch.empty(B, H, Kg, **i32))


@torch.library.custom_op("hga::attend_decode", mutates_args=())
def attend_decode(pi: List[int], pf: List[float], q: Tensor, seq_pos: Tensor, hot_k: Tensor, hot_v: Tensor,
                  hot_mode: int, cold_k: Optional[Tensor], cold_v: Optional[Tensor], open_gid: Tensor,
                  open_t0: Tensor) -> Tensor:
    return ops.attend_decode(_params(pi, pf), q, seq_pos, hot_k, hot_v, hot_mode, cold_k, cold_v, open_gid, open_t0)


@attend_decode.register_fake
def _(pi, pf, q, seq_pos, hot_k, hot_v, hot_mode, cold_k, cold_v, open_gid, open_t0):
    return torch.empty_like(q)


@torch.library.custom_op("hga::attend_decode_dca", mutates_args=())
def attend_decode_dca(pi: List[int], pf: List[float], q: Tensor, seq_pos: Tensor, hot_k: Tensor, hot_v: Tensor,
                      hot_mode: int, cold_k: Optional[Tensor], cold_v: Optional[Tensor], open_gid: Tensor,
                      open_t0: Tensor, open_pos: Optional[Tensor], dca_chunk: int, dca_ceil: int,
                      theta: float) -> Tensor:
    return ops.attend_decode_dca(_params(pi, pf), q, seq_pos, hot_k, hot_v, hot_mode, cold_k, cold_v, open_gid,
                                 open_t0, dca_chunk, dca_ceil, theta, open_pos=open_pos)


@attend_decode_dca.register_fake
def _(pi, pf, q, seq_pos, hot_k, hot_v, hot_mode, cold_k, cold_v, open_gid, open_t0, open_pos, dca_chunk, dca_ceil,
      theta):
    return torch.empty_like(q)


@torch.library.custom_op("hga::gather_h2d", mutates_args=("bank_k", "bank_v", "slot_gid", "gid_slot", "slot_stamp",
                                                          "counters"))
def gather_h2d(pi: List[int], pf: List[float], open_gid: Tensor, rec_k: Tensor, rec_v: Tensor, bank_k: Tensor,
               bank_v: Tensor, slot_gid: Tensor, gid_slot: Tensor, slot_stamp: Tensor, stamp: int,
               counters: Tensor) -> Tensor:
    return ops.gather_h2d(_params(pi, pf), open_gid, rec_k, rec_v, bank_k, bank_v, slot_gid, gid_slot, slot_stamp,
                          stamp, counters)


@gather_h2d.register_fake
def _(pi, pf, open_gid, rec_k, rec_v, bank_k, bank_v, slot_gid, gid_slot, slot_stamp, stamp, counters):
    return torch.empty_like(open_gid)
