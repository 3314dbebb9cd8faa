"""Tensor-level wrappers of the C ABI (device tensors in, device tensors out).

Every function validates shapes / dtypes / devices, allocates its outputs through PyTorch's
caching allocator and launches on the current CUDA stream.  Tensors must live on a CUDA device:
there is no CPU path.
"""
from __future__ import annotations

from typing import Dict, Optional, Tuple

import torch

from . import _lib
from ._lib import HgaParams, check, lib, ptr, stream_ptr

Q_BHSD, Q_BSHD = 0, 1


def _require_cuda(*ts):
    for t in ts:
        if t is not None and t.device.type != "cuda":
            raise _lib.HgaError("hga ops run on CUDA tensors only (no CPU fallback); got device "
                                f"{t.device}")


def route_sizes(p: HgaParams, seq_len: int) -> Tuple[int, int, int, int]:
    """(N, Kc, Kg, Kg_request) exactly as vectorized.py:304, 365-366 size them."""
    C = p.chunk_size
    M = C // p.group_size
    N = (seq_len + C - 1) // C
    Kc = min(p.topk_chunks, N) if p.topk_chunks > 0 else 0
    Tg = Kc * M
    Kg = min(p.topk_groups, Tg) if p.topk_groups > 0 else 0
    Kgr = min(p.topk_groups // 2, Tg) if p.topk_groups > 0 else 0
    if Kgr == 0:
        Kg = 0
    return N, Kc, Kg, Kgr


def q_view(q: torch.Tensor) -> Tuple[torch.Tensor, int]:
    """(q, layout): 0 for a contiguous [B,H,S,Dh] tensor, 1 for a [B,H,S,Dh] view of a contiguous
    [B,S,H,Dh]; any other strided view is made contiguous first."""
    if q.is_contiguous():
        return q, Q_BHSD
    if q.transpose(1, 2).is_contiguous():
        return q, Q_BSHD
    return q.contiguous(), Q_BHSD


def kv_cap_of(t: torch.Tensor) -> int:
    """Rows allocated per (batch, kv-head) of a [B,KVH,S,Dh] view into a [B,KVH,cap,Dh] buffer."""
    B, KVH, S, Dh = t.shape
    if t.stride(3) != 1 or t.stride(2) != Dh or t.stride(1) % Dh or t.stride(0) != KVH * t.stride(1):
        raise _lib.HgaError(f"K/V tensor must be a row-slice of a contiguous [B,KVH,cap,Dh] buffer; strides {t.stride()}")
    return t.stride(1) // Dh


def summaries(p: HgaParams, k_raw: torch.Tensor, k_rope: torch.Tensor, v: torch.Tensor,
              cos: torch.Tensor, sin: torch.Tensor, *, seq_len: Optional[int] = None, pos0: int = 0,
              rot_row0: int = 0, out: Optional[Tuple[torch.Tensor, torch.Tensor, torch.Tensor]] = None,
              out_chunk0: int = 0, with_group_v: bool = True, round_table: bool = False):
    """Chunk / group summaries of k_* [B,KVH,S,Dh] (see hga_summaries).  cos/sin [R, Dh].

    Returns (chunk_k [B,KVH,N,Dh], group_k [B,KVH,N,M,Dh], group_v or None), or fills ``out``
    (capacity buffers, chunk slots [out_chunk0, out_chunk0+N)).  ``round_table`` rounds an fp32
    table to the model dtype at use (the chunk-parallel path's ``cos.to(x.dtype)``).
    """
    _require_cuda(k_raw, k_rope, v, cos, sin)
    B, KVH, S, Dh = k_raw.shape
    S = S if seq_len is None else seq_len
    C = p.chunk_size
    M = C // p.group_size
    N = (S + C - 1) // C
    cap = kv_cap_of(k_raw)
    if kv_cap_of(k_rope) != cap or kv_cap_of(v) != cap:
        raise _lib.HgaError("k_raw / k_rope / v must share one capacity layout")
    for t in (k_rope, v):
        if t.dtype != k_raw.dtype:
            raise _lib.HgaError("k_raw / k_rope / v dtypes differ")
    if cos.dtype not in (torch.float32, k_raw.dtype) or sin.dtype != cos.dtype:
        raise _lib.HgaError("cos/sin must be fp32 or the model dtype")
    cos, sin = cos.contiguous(), sin.contiguous()
    if out is None:
        ck = torch.empty(B, KVH, N, Dh, device=k_raw.device, dtype=k_raw.dtype)
        gk = torch.empty(B, KVH, N, M, Dh, device=k_raw.device, dtype=k_raw.dtype)
        gv = torch.empty_like(gk) if with_group_v else None
        sum_cap = N
    else:
        ck, gk, gv = out
        sum_cap = ck.shape[2]
    if cos.dtype == torch.float32 and k_raw.dtype != torch.float32:
        rot_mode = _lib.ROT_F32_ROUNDED if round_table else _lib.ROT_F32
    else:
        rot_mode = _lib.ROT_MODEL if cos.dtype != torch.float32 else _lib.ROT_F32
    check(lib().hga_summaries(ctypes_params(p), S, pos0, ptr(k_raw), ptr(k_rope), ptr(v), cap, ptr(cos), ptr(sin),
                              rot_mode, rot_row0, ptr(ck), ptr(gk), ptr(gv), sum_cap, out_chunk0,
                              stream_ptr(k_raw.device)), "hga_summaries")
    return ck, gk, gv


def summaries_dual_supported(p: HgaParams) -> bool:
    """hga_summaries_dual's shape rule: bf16/fp16, head_dim 64 or 128, chunk and group sizes multiples
    of 16 (chunk <= 128)."""
    return (p.dtype in (_lib.DTYPE_CODE[torch.bfloat16], _lib.DTYPE_CODE[torch.float16]) and p.head_dim in (64, 128)
            and p.chunk_size % 16 == 0 and p.group_size % 16 == 0 and p.chunk_size <= 128)


def summaries_dual(p: HgaParams, k_raw: torch.Tensor, k_rope: torch.Tensor, v: torch.Tensor,
                   cos_a: torch.Tensor, sin_a: torch.Tensor, cos_b: torch.Tensor, sin_b: torch.Tensor,
                   out_b: Tuple[torch.Tensor, torch.Tensor, Optional[torch.Tensor]], n_b: int, *,
                   round_a: bool = True, rot_row0_a: int = 0, rot_row0_b: int = 0):
    """Routing summaries (set A, fresh [B,KVH,N,(M,)Dh] tensors; fp32 table A, entries rounded to the
    model dtype when ``round_a``) and the store seed of the first ``n_b`` closed chunks (set B, into
    the capacity buffers ``out_b``; fp32 table B) from one read of K/V (see hga_summaries_dual).
    Returns (chunk_k, group_k) of set A."""
    _require_cuda(k_raw, k_rope, v, cos_a, sin_a, cos_b, sin_b)
    B, KVH, S, Dh = k_raw.shape
    C = p.chunk_size
    M = C // p.group_size
    N = (S + C - 1) // C
    cap = kv_cap_of(k_raw)
    if kv_cap_of(k_rope) != cap or kv_cap_of(v) != cap:
        raise _lib.HgaError("k_raw / k_rope / v must share one capacity layout")
    for t in (cos_a, sin_a, cos_b, sin_b):
        if t.dtype != torch.float32:
            raise _lib.HgaError("summaries_dual takes fp32 rotary tables")
    cos_a, sin_a, cos_b, sin_b = (t.contiguous() for t in (cos_a, sin_a, cos_b, sin_b))
    ck = torch.empty(B, KVH, N, Dh, device=k_raw.device, dtype=k_raw.dtype)
    gk = torch.empty(B, KVH, N, M, Dh, device=k_raw.device, dtype=k_raw.dtype)
    ckb, gkb, gvb = out_b
    check(lib().hga_summaries_dual(ctypes_params(p), S, 0, ptr(k_raw), ptr(k_rope), ptr(v), cap, ptr(cos_a), ptr(sin_a),
                                   rot_row0_a, int(round_a), ptr(ck), ptr(gk), N, 0, ptr(cos_b), ptr(sin_b), rot_row0_b,
                                   n_b, ptr(ckb), ptr(gkb), ptr(gvb), ckb.shape[2], 0, stream_ptr(k_raw.device)),
          "hga_summaries_dual")
    return ck, gk


def ctypes_params(p: HgaParams):
    import ctypes
    return ctypes.byref(p)


def route_prefill(p: HgaParams, q: torch.Tensor, chunk_k: torch.Tensor, group_k: torch.Tensor,
                  seq_len: Optional[int] = None, debug: bool = False, impl: int = 0,
                  chunk_range: Optional[Tuple[int, int]] = None) -> Dict[str, torch.Tensor]:
    """Two-level prefill routing (see hga_route_prefill_impl).  q [B,H,S,Dh] (or a BSHD view).
    impl: 0 auto, 1 portable SIMT router, 2 tcgen05 router.  ``chunk_range=(lo, hi)`` routes only
    query chunks [lo, hi) of a ``seq_len``-token sequence: q then holds just those chunks' rows and
    the lists are [B,H,hi-lo,K] (hga_route_prefill_range)."""
    _require_cuda(q, chunk_k, group_k)
    B, H, S, Dh = q.shape
    S = S if seq_len is None else seq_len
    N, Kc, Kg, _ = route_sizes(p, S)
    lo, hi = (0, N) if chunk_range is None else chunk_range
    NL = hi - lo
    dev = q.device
    C = p.chunk_size
    M = C // p.group_size
    res = {
        "sel_chunk": torch.empty(B, H, NL, Kc, device=dev, dtype=torch.int32),
        "sel_t0": torch.empty(B, H, NL, Kc, device=dev, dtype=torch.int32),
        "open_gid": torch.empty(B, H, NL, Kg, device=dev, dtype=torch.int32),
        "open_t0": torch.empty(B, H, NL, Kg, device=dev, dtype=torch.int32),
    }
    if debug:
        res["dbg_l1"] = torch.full((B, H, NL, C, N), float("nan"), device=dev, dtype=torch.float32)
        res["dbg_l2"] = torch.full((B, H, NL, C, Kc * M), float("nan"), device=dev, dtype=torch.float32)
    sum_cap = chunk_k.stride(1) // Dh
    if (chunk_k.stride(-1) != 1 or chunk_k.stride(2) != Dh or group_k.stride(-1) != 1
            or group_k.stride(1) != sum_cap * M * Dh or chunk_k.stride(0) != chunk_k.shape[1] * chunk_k.stride(1)):
        raise _lib.HgaError("summaries must be row-slices of contiguous [B,KVH,cap,(M,)Dh] buffers")
    q, q_layout = q_view(q)
    check(lib().hga_route_prefill_range(ctypes_params(p), S, lo, hi, ptr(q), q_layout, ptr(chunk_k), ptr(group_k),
                                        sum_cap, ptr(res["sel_chunk"]), ptr(res["sel_t0"]), ptr(res["open_gid"]),
                                        ptr(res["open_t0"]), ptr(res.get("dbg_l1")), ptr(res.get("dbg_l2")), impl,
                                        stream_ptr(dev)), "hga_route_prefill")
    return res


def attend_prefill(p: HgaParams, q: torch.Tensor, k_rope: torch.Tensor, v: torch.Tensor,
                   open_gid: torch.Tensor, open_t0: torch.Tensor, seq_len: Optional[int] = None,
                   out_layout: int = Q_BSHD, impl: int = 0, out: Optional[torch.Tensor] = None,
                   chunk_range: Optional[Tuple[int, int]] = None) -> torch.Tensor:
    """Working-set attention (see hga_attend_prefill).  Returns [B,H,S,Dh] (a view of a BSHD
    buffer when out_layout == 1).  ``chunk_range=(lo, hi)`` attends only query chunks [lo, hi) of
    a ``seq_len``-token sequence (q, lists and out hold just those chunks; hga_attend_prefill_range)."""
    _require_cuda(q, k_rope, v, open_gid, open_t0)
    B, H, SQ, Dh = q.shape
    S = SQ if seq_len is None else seq_len
    C = p.chunk_size
    lo, hi = (0, (S + C - 1) // C) if chunk_range is None else chunk_range
    SQ = min(S, hi * C) - lo * C
    cap = kv_cap_of(k_rope)
    if kv_cap_of(v) != cap:
        raise _lib.HgaError("k_rope and v must share one capacity layout")
    if out is None:
        if out_layout == Q_BSHD:
            out = torch.empty(B, SQ, H, Dh, device=q.device, dtype=q.dtype)
        else:
            out = torch.empty(B, H, SQ, Dh, device=q.device, dtype=q.dtype)
    q, q_layout = q_view(q)
    check(lib().hga_attend_prefill_range(ctypes_params(p), S, lo, hi, ptr(q), q_layout, ptr(k_rope), ptr(v), cap,
                                         ptr(open_gid), ptr(open_t0), ptr(out), out_layout, impl,
                                         stream_ptr(q.device)), "hga_attend_prefill")
    return out.transpose(1, 2) if out_layout == Q_BSHD else out


def qkv_prologue(p: HgaParams, qkv: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, *,
                 q_norm_w: Optional[torch.Tensor] = None, k_norm_w: Optional[torch.Tensor] = None,
                 eps: float = 1e-6, norm_mode: int = 0, rope_mode: int = 0, rot_row0: int = 0, pos0: int = 0,
                 kv_out: Optional[Tuple[torch.Tensor, torch.Tensor, torch.Tensor]] = None, kv_row0: int = 0):
    """Fused q/k RMSNorm + RoPE + layout (see hga_qkv_prologue).

    qkv [B, S, (H + 2*KVH) * Dh] (a fused projection output).  Returns (q_rope [B,H,S,Dh] view of a
    [B,S,H,Dh] buffer, k_raw, k_rope, v [B,KVH,S,Dh] row-slices of the kv_out buffers or fresh
    tensors)."""
    _require_cuda(qkv, cos, sin)
    B, S, W = qkv.shape
    H, KVH, Dh = p.nhead, p.kv_heads, p.head_dim
    if qkv.stride(2) != 1 or (B > 1 and qkv.stride(0) != S * qkv.stride(1)):
        raise _lib.HgaError("qkv must be contiguous in its token rows")
    row_stride = qkv.stride(1)
    if W < (H + 2 * KVH) * Dh:
        raise _lib.HgaError("qkv rows are narrower than (H + 2*KVH) * Dh")
    want_rope_dtype = torch.float32 if rope_mode == 0 else qkv.dtype
    if cos.dtype != want_rope_dtype or sin.dtype != want_rope_dtype:
        raise _lib.HgaError(f"rope_mode {rope_mode} needs a {want_rope_dtype} table")
    cos, sin = cos.contiguous(), sin.contiguous()
    dev = qkv.device
    q = torch.empty(B, S, H, Dh, device=dev, dtype=qkv.dtype)
    if kv_out is None:
        kraw = torch.empty(B, KVH, S, Dh, device=dev, dtype=qkv.dtype)
        krope = torch.empty_like(kraw)
        v = torch.empty_like(kraw)
        cap = S
    else:
        kraw, krope, v = kv_out
        cap = kv_cap_of(kraw)
    for w in (q_norm_w, k_norm_w):
        if w is not None and (w.numel() != Dh or w.dtype != qkv.dtype or not w.is_contiguous()):
            raise _lib.HgaError("norm weights must be contiguous [Dh] tensors in the model dtype")
    check(lib().hga_qkv_prologue(ctypes_params(p), S, ptr(qkv), row_stride, ptr(q_norm_w), ptr(k_norm_w), float(eps),
                                 norm_mode, ptr(cos), ptr(sin), rope_mode, rot_row0, pos0, ptr(q), ptr(kraw),
                                 ptr(krope), ptr(v), cap, kv_row0, stream_ptr(dev)), "hga_qkv_prologue")
    if kv_out is not None:
        sl = slice(kv_row0, kv_row0 + S)
        return q.transpose(1, 2), kraw[:, :, sl], krope[:, :, sl], v[:, :, sl]
    return q.transpose(1, 2), kraw, krope, v


# ---------------------------------------------------------------------------------------------
# incremental decode
# ---------------------------------------------------------------------------------------------
def decode_sizes(p: HgaParams, nmid_max: int) -> Tuple[int, int]:
    """(Kc, Kg) of a decode block whose largest routed pool is nmid_max (chunk_router.py:226, 256)."""
    M = p.chunk_size // p.group_size
    Kc = min(p.topk_chunks, nmid_max) if p.topk_chunks > 0 else 0
    Kg = min(p.topk_groups, Kc * M) if p.topk_groups > 0 else 0
    return Kc, Kg


def route_decode(p: HgaParams, q: torch.Tensor, seq_pos: torch.Tensor, chunk_k: torch.Tensor,
                 group_k: torch.Tensor, nmid_max: int, impl: int = 0) -> Dict[str, torch.Tensor]:
    """Routing of one decode block (see hga_route_decode_impl).  q [B,H,L,Dh] contiguous.
    impl: 0 auto, 1 portable kernel, 2 single-token kernel."""
    _require_cuda(q, seq_pos, chunk_k, group_k)
    B, H, L, Dh = q.shape
    Kc, Kg = decode_sizes(p, nmid_max)
    dev = q.device
    res = {"mid_chunk": torch.empty(B, H, Kc, device=dev, dtype=torch.int32),
           "mid_t0": torch.empty(B, H, Kc, device=dev, dtype=torch.int32),
           "open_gid": torch.empty(B, H, Kg, device=dev, dtype=torch.int32),
           "open_t0": torch.empty(B, H, Kg, device=dev, dtype=torch.int32)}
    if not q.is_contiguous():
        q = q.contiguous()
    sum_cap = chunk_k.stride(1) // Dh
    check(lib().hga_route_decode_impl(ctypes_params(p), L, ptr(q), ptr(seq_pos), ptr(chunk_k), ptr(group_k),
                                      sum_cap, nmid_max, ptr(res["mid_chunk"]), ptr(res["mid_t0"]),
                                      ptr(res["open_gid"]), ptr(res["open_t0"]), impl, stream_ptr(dev)),
          "hga_route_decode")
    return res


def attend_decode(p: HgaParams, q: torch.Tensor, seq_pos: torch.Tensor, hot_k: torch.Tensor, hot_v: torch.Tensor,
                  hot_mode: int, cold_k: Optional[torch.Tensor], cold_v: Optional[torch.Tensor],
                  open_gid: torch.Tensor, open_t0: torch.Tensor, out: Optional[torch.Tensor] = None,
                  impl: int = 0) -> torch.Tensor:
    """Attention of one decode block (see hga_attend_decode_impl).  Returns [B,H,L,Dh].
    impl: 0 auto, 1 portable kernel, 2 short-block kernel."""
    _require_cuda(q, seq_pos, hot_k, hot_v, open_gid, open_t0)
    if not q.is_contiguous():
        q = q.contiguous()
    B, H, L, Dh = q.shape
    out = torch.empty_like(q) if out is None else out
    hot_cap = kv_cap_of(hot_k)
    cold_cap = kv_cap_of(cold_k) if cold_k is not None else hot_cap
    Kg = open_gid.shape[-1]
    check(lib().hga_attend_decode_impl(ctypes_params(p), L, ptr(q), ptr(seq_pos), ptr(hot_k), ptr(hot_v), hot_cap,
                                       hot_mode, ptr(cold_k), ptr(cold_v), cold_cap, ptr(open_gid), ptr(open_t0), Kg,
                                       ptr(out), impl, stream_ptr(q.device)), "hga_attend_decode")
    return out


def dca_rope_table(dca_ceil: int, head_dim: int, theta: float, device) -> Tuple[torch.Tensor, torch.Tensor]:
    """fp32 rotate-half RoPE cos / sin [dca_ceil + 1, Dh] of positions 0..dca_ceil, evaluated like
    the Qwen3 wrapper's _dca_rope (qwen_routed_attention.py:66-81) in fp32 on the host (torch's
    CPU cos / sin, so the rows are the same on every device), then copied to ``device`` and cached."""
    key = (str(device), int(dca_ceil), int(head_dim), float(theta))
    t = _DCA_TABLES.get(key)
    if t is None:
        half = head_dim // 2
        inv = 1.0 / (theta ** (torch.arange(half, dtype=torch.float32) / half))
        f = torch.arange(dca_ceil + 1, dtype=torch.float32).unsqueeze(-1) * inv
        emb = torch.cat((f, f), dim=-1)
        t = (emb.cos().to(device).contiguous(), emb.sin().to(device).contiguous())
        _DCA_TABLES[key] = t
    return t


_DCA_TABLES: dict = {}


def attend_decode_dca(p: HgaParams, q: torch.Tensor, seq_pos: torch.Tensor, hot_k: torch.Tensor, hot_v: torch.Tensor,
                      hot_mode: int, cold_k: Optional[torch.Tensor], cold_v: Optional[torch.Tensor],
                      open_gid: torch.Tensor, open_t0: torch.Tensor, dca_chunk: int, dca_ceil: int, theta: float,
                      open_pos: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Dual Chunk Attention of one decode block (see hga_attend_decode_dca): q [B,H,L,Dh] un-roped;
    the store holds the intra-chunk-roped keys.  Returns [B,H,L,Dh]."""
    _require_cuda(q, seq_pos, hot_k, hot_v, open_gid, open_t0)
    q = q.contiguous()
    B, H, L, Dh = q.shape
    out = torch.empty_like(q) if out is None else out
    cos, sin = dca_rope_table(dca_ceil, Dh, theta, q.device)
    hot_cap = kv_cap_of(hot_k)
    cold_cap = kv_cap_of(cold_k) if cold_k is not None else hot_cap
    Kg = open_gid.shape[-1]
    check(lib().hga_attend_decode_dca(ctypes_params(p), L, ptr(q), ptr(seq_pos), ptr(hot_k), ptr(hot_v), hot_cap,
                                      hot_mode, ptr(cold_k), ptr(cold_v), cold_cap, ptr(open_gid), ptr(open_t0),
                                      ptr(open_pos.contiguous()) if open_pos is not None else None, Kg, ptr(cos),
                                      ptr(sin), int(dca_chunk), int(dca_ceil), ptr(out), stream_ptr(q.device)),
          "hga_attend_decode_dca")
    return out


def gather_h2d(p: HgaParams, open_gid: torch.Tensor, rec_k: torch.Tensor, rec_v: torch.Tensor, bank_k: torch.Tensor,
               bank_v: torch.Tensor, slot_gid: torch.Tensor, gid_slot: torch.Tensor, slot_stamp: torch.Tensor,
               stamp: int, counters: Optional[torch.Tensor] = None) -> torch.Tensor:
    """One step of the RAM tier's VRAM token bank (see hga_gather_h2d).  open_gid [B,H,Kg] int32;
    rec_* [B,KVH,rec_cap,Dh] (pinned host or device); bank_* [B,KVH,slots*group_size,Dh]; maps as
    documented in the header; counters int64 [2] (hits, misses) or None.  Returns open_slot
    [B,H,Kg] (bank slots of the entries, -1 padding)."""
    _require_cuda(open_gid, bank_k, bank_v, slot_gid, gid_slot, slot_stamp)
    B, H, Kg = open_gid.shape
    open_gid = open_gid.contiguous()
    out = torch.empty_like(open_gid)
    check(lib().hga_gather_h2d(ctypes_params(p), ptr(open_gid), Kg, ptr(rec_k), ptr(rec_v), kv_cap_of(rec_k), ptr(bank_k),
                               ptr(bank_v), slot_gid.shape[2], ptr(slot_gid), ptr(gid_slot), gid_slot.shape[2],
                               ptr(slot_stamp), int(stamp), ptr(out), ptr(counters), stream_ptr(open_gid.device)),
          "hga_gather_h2d")
    return out


def append_tokens(p: HgaParams, seq_pos: torch.Tensor, k_rope: torch.Tensor, v: torch.Tensor,
                  k_raw: Optional[torch.Tensor], hot_k: torch.Tensor, hot_v: torch.Tensor, hot_mode: int,
                  cold_k: Optional[torch.Tensor], cold_v: Optional[torch.Tensor],
                  active_raw: Optional[torch.Tensor]) -> None:
    """Write a block's new K/V rows (see hga_append_tokens).  k_rope/v/k_raw [B,KVH,L,Dh]."""
    _require_cuda(seq_pos, k_rope, v, hot_k, hot_v)
    k_rope, v = k_rope.contiguous(), v.contiguous()
    k_raw = None if k_raw is None else k_raw.contiguous()
    L = k_rope.shape[2]
    check(lib().hga_append_tokens(ctypes_params(p), L, ptr(seq_pos), ptr(k_rope), ptr(v), ptr(k_raw), ptr(hot_k),
                                  ptr(hot_v), kv_cap_of(hot_k), hot_mode, ptr(cold_k), ptr(cold_v),
                                  kv_cap_of(cold_k) if cold_k is not None else 0, ptr(active_raw),
                                  stream_ptr(k_rope.device)), "hga_append_tokens")


def shard_unpack(recv: torch.Tensor, rank_stride: int, part_offset: int, world: int, pieces: int,
                 dst_block, bk: int, rows: int, row_bytes: int, dst: torch.Tensor) -> None:
    """Scatter one part of an all-gathered multi-GPU prefill buffer into sequence order (see
    hga_shard_unpack; strides and offsets in bytes, ``dst_block`` a list of world*pieces ints)."""
    import ctypes
    _require_cuda(recv, dst)
    table = (ctypes.c_int32 * len(dst_block))(*dst_block)
    check(lib().hga_shard_unpack(ptr(recv), rank_stride, part_offset, world, pieces,
                                 ctypes.cast(table, ctypes.c_void_p), bk, rows, row_bytes,
                                 ptr(dst), stream_ptr(dst.device)), "hga_shard_unpack")
