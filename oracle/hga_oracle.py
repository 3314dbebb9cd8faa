"""CPU oracle for the HGA routed-attention hot path.  TEST INFRASTRUCTURE ONLY.

This module is the checker the CUDA path is compared against.  Only ``tests/``,
``__graft_entry__.smoke()`` and the ``cpu_baseline`` / ``--impl reference`` legs of
``bench.py`` may import it; the product package never does.

It restates, one query chunk at a time (so 32K/131K sequences fit in host RAM), the
reference's chunk-parallel prefill path and its default attention:

* summary builder ......... ExistingModelFineTuning/KvRouter/vectorized.py:146-183, 233-287
* store seed summaries .... ExistingModelFineTuning/KvRouter/chunk_router.py:553-599, 693-735
* chunk router (level 1) .. vectorized.py:99-140, 296-337
* group router (level 2) .. vectorized.py:339-384
* working-set assembly .... vectorized.py:386-490
* attention ............... ExistingModelFineTuning/KvRouter/chunk_router.py:139-162

and the incremental single-chunk decode path:

* route decision .......... chunk_router.py:188-277
* decode segments ......... chunk_router.py:279-407

The arithmetic is done with the same torch CPU operators, dtypes and rounding points as
the reference (bf16 score tensors rounded before and after the softmax scale, fp32
attention), so on identical inputs it reproduces the reference's selections.  Its routing
decisions are reported in the compact form the CUDA path emits: per (batch, head, query
chunk) the selected chunks / opened groups and, for each, ``t0`` = the first query row of
the chunk that can see it (``chunk_size`` = never).  Visibility in the reference is a
cumulative OR over query rows, so ``t0`` carries the whole mask.

Pinned against the reference itself: ``tests/golden/make_golden.py`` runs the unmodified
reference on seeded inputs and stores its outputs; ``tests/test_oracle_golden.py`` checks this
restatement against them.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Dict, Optional

import torch

NEG = -1.0e4  # the reference's finite mask fill (vectorized.py:38, chunk_router.py:55)


@dataclass
class OracleParams:
    nhead: int
    kv_heads: int
    head_dim: int
    chunk_size: int = 64
    group_size: int = 16
    topk_chunks: int = 20
    topk_groups: int = 32
    keep_first: int = 0
    keep_last: int = 0
    theta: float = 1_000_000.0
    mixed_rope_threshold: float = 0.5
    mixed_rope_cutoff_pair: Optional[int] = None

    @property
    def M(self) -> int:
        return self.chunk_size // self.group_size

    @property
    def rep(self) -> int:
        return self.nhead // self.kv_heads

    @property
    def scale(self) -> float:
        return self.head_dim ** -0.5

    @property
    def group_kv_scale(self) -> float:
        return 1.0 / (self.group_size + math.sqrt(self.group_size))


# ---------------------------------------------------------------------------------------------
# summaries
# ---------------------------------------------------------------------------------------------
def mixed_cutoff_pair(p: OracleParams) -> int:
    """Number of RoPE pairs taken token-wise (vectorized.py:146-155)."""
    half = p.head_dim // 2
    if p.mixed_rope_cutoff_pair is not None:
        return int(p.mixed_rope_cutoff_pair)
    cutoff = 0
    for i in range(half):
        inv_freq = 1.0 / (p.theta ** (i / half))
        if max(1, p.chunk_size - 1) * inv_freq > p.mixed_rope_threshold:
            cutoff = i + 1
    return cutoff


def _rotate(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    half = x.shape[-1] // 2
    return x * cos + torch.cat((-x[..., half:], x[..., :half]), dim=-1) * sin


def _summary(p, raw, rope, reduce_dim, anchor_cos, anchor_sin, scale):
    """Mixed-RoPE summary: vectorized.py:168-183 (masking already applied by the caller)."""
    raw_sum = raw.sum(dim=reduce_dim) * scale
    endpoint = _rotate(raw_sum.float(), anchor_cos, anchor_sin).to(raw_sum.dtype)
    tokenwise = rope.sum(dim=reduce_dim) * scale
    half = p.head_dim // 2
    keep = torch.arange(half) < mixed_cutoff_pair(p)
    keep = torch.cat([keep, keep])
    return torch.where(keep, tokenwise, endpoint)


def rope_table(theta: float, head_dim: int, positions: torch.Tensor):
    """fp32 cos/sin rows for ``positions`` (chunk_router.py:702-709)."""
    half = head_dim // 2
    inv = 1.0 / (theta ** (torch.arange(half, dtype=torch.float32) / half))
    f = positions.to(torch.float32).unsqueeze(-1) * inv
    emb = torch.cat((f, f), dim=-1)
    return emb.cos(), emb.sin()


def summaries_prefill(p: OracleParams, k_raw, k_rope, v, cos, sin):
    """Routing summaries of the chunk-parallel path at KV-head granularity.

    k_raw/k_rope/v ``[B, KVH, S, Dh]``; cos/sin ``[S, Dh]`` (the table the caller hands the
    router, already in the model dtype).  Returns chunk_k ``[B,KVH,N,Dh]``, group_k and
    group_v ``[B,KVH,N,M,Dh]`` (vectorized.py:233-287; the reference computes the same values
    once per query head after ``repeat_interleave``).
    """
    B, KVH, S, Dh = k_raw.shape
    C, gs, M = p.chunk_size, p.group_size, p.M
    dtype = k_raw.dtype
    N = (S + C - 1) // C
    pad = N * C - S

    def padded(x):
        return torch.cat([x, x.new_zeros(B, KVH, pad, Dh)], dim=2) if pad else x

    valid = (torch.arange(N * C) < S).view(N, C)
    chunk_len = valid.sum(1)
    c_mid = (torch.arange(N) * C + (chunk_len.clamp_min(1) - 1) // 2).clamp_max(S - 1)
    g_len = valid.view(N, M, gs).sum(-1)
    g_start = torch.arange(N)[:, None] * C + torch.arange(M)[None, :] * gs
    g_mid = (g_start + (g_len.clamp_min(1) - 1) // 2).clamp_max(S - 1)

    raw = padded(k_raw).reshape(B, KVH, N, C, Dh)
    rope = padded(k_rope).reshape(B, KVH, N, C, Dh)
    vv = padded(v).reshape(B, KVH, N, C, Dh)
    cmask = valid.view(1, 1, N, C, 1).to(dtype)
    chunk_k = _summary(p, raw * cmask, rope * cmask, 3, cos[c_mid].view(1, 1, N, Dh),
                       sin[c_mid].view(1, 1, N, Dh), 1.0)
    gmask = valid.view(1, 1, N, M, gs, 1).to(dtype)
    graw = raw.reshape(B, KVH, N, M, gs, Dh) * gmask
    grope = rope.reshape(B, KVH, N, M, gs, Dh) * gmask
    group_k = _summary(p, graw, grope, 4, cos[g_mid].view(1, 1, N, M, Dh),
                       sin[g_mid].view(1, 1, N, M, Dh), p.group_kv_scale)
    group_v = (vv.reshape(B, KVH, N, M, gs, Dh) * gmask).sum(dim=4) * p.group_kv_scale
    return chunk_k, group_k, group_v


def summaries_store(p: OracleParams, k_raw, k_rope, v, first_chunk: int = 0):
    """Summaries of complete chunks as handed to the store (chunk_router.py:563-587, 631-657).

    Anchors are fixed at ``(len-1)//2`` and the rotary rows are recomputed in fp32 from theta.
    ``k_*`` cover whole chunks starting at chunk ``first_chunk``.
    """
    B, KVH, S, Dh = k_raw.shape
    C, gs, M = p.chunk_size, p.group_size, p.M
    n = S // C
    raw = k_raw[:, :, : n * C].reshape(B, KVH, n, C, Dh)
    rope = k_rope[:, :, : n * C].reshape(B, KVH, n, C, Dh)
    vv = v[:, :, : n * C].reshape(B, KVH, n, C, Dh)
    ar = torch.arange(first_chunk, first_chunk + n)
    g_anchor = ar[:, None] * C + torch.arange(M)[None, :] * gs + (gs - 1) // 2
    gc, gsn = rope_table(p.theta, Dh, g_anchor)
    group_k = _summary(p, raw.reshape(B, KVH, n, M, gs, Dh), rope.reshape(B, KVH, n, M, gs, Dh), 4,
                       gc.view(1, 1, n, M, Dh), gsn.view(1, 1, n, M, Dh), p.group_kv_scale)
    group_v = vv.reshape(B, KVH, n, M, gs, Dh).sum(dim=4) * p.group_kv_scale
    cc, cs = rope_table(p.theta, Dh, ar * C + (C - 1) // 2)
    chunk_k = _summary(p, raw, rope, 3, cc.view(1, 1, n, Dh), cs.view(1, 1, n, Dh), 1.0)
    return chunk_k, group_k, group_v


# ---------------------------------------------------------------------------------------------
# near-tie bookkeeping
# ---------------------------------------------------------------------------------------------
# Two implementations that accumulate the same q.k dot product in fp32 in a different order
# can disagree by a few units of 2^-24 * sum|q_i k_i|.  After the bf16 rounding points of the
# reference that becomes a disagreement of one bf16 unit, and torch.topk's order among EQUAL
# scores is implementation-defined.  A selection therefore "depends on a near tie" when a
# selected and an unselected candidate have overlapping possible-score intervals.  The interval
# of each score is computed from an fp64 dot product widened by an fp32 accumulation bound.
_ACC_BOUND = 2.0 ** -22


def score_bounds(q: torch.Tensor, k: torch.Tensor, scale: float, dtype: torch.dtype, eq: str,
                 acc: float = _ACC_BOUND):
    """Possible-score interval (lo, hi) as fp64 for ``einsum(eq, q, k) * scale`` in ``dtype``.

    ``acc`` is the relative accumulation bound (times sqrt(Dh) * sum|q_i k_i|); ``acc=0`` gives the
    exactly rounded score."""
    qd, kd = q.double(), k.double()
    d = torch.einsum(eq, qd, kd)
    e = torch.einsum(eq, qd.abs(), kd.abs()) * (acc * math.sqrt(q.shape[-1]))
    if dtype in (torch.bfloat16, torch.float16):
        lo = ((d - e).to(dtype).float() * scale).to(dtype).double()
        hi = ((d + e).to(dtype).float() * scale).to(dtype).double()
    else:
        lo, hi = (d - e) * scale, (d + e) * scale
    return lo, hi


def _set_tie(lo, hi, selected, real, resolved: bool = False):
    """True where a selected real candidate could score <= an unselected real one.

    ``resolved``: equal scores are ordered by a fixed rule shared by both implementations (the
    ``"index"`` tie rule), so a selected and an unselected candidate whose intervals are the SAME
    single point are not ambiguous; only intervals that span a rounding boundary are."""
    big = torch.finfo(torch.float64).max
    s_m, u_m = selected & real, ~selected & real
    sel_lo = torch.where(s_m, lo, torch.full_like(lo, big)).min(dim=-1).values
    rest_hi = torch.where(u_m, hi, torch.full_like(hi, -big)).max(dim=-1).values
    if not resolved:
        return sel_lo <= rest_hi
    wide = hi != lo
    s_wide = (s_m & (lo == sel_lo.unsqueeze(-1)) & wide).any(-1)
    u_wide = (u_m & (hi == rest_hi.unsqueeze(-1)) & wide).any(-1)
    return (sel_lo < rest_hi) | ((sel_lo == rest_hi) & (s_wide | u_wide))


def _pair_ambiguous(lo_a, hi_a, lo_b, hi_b, resolved: bool):
    """Elementwise: could a score in [lo_a, hi_a] rank at or below one in [lo_b, hi_b]?"""
    amb = lo_a <= hi_b
    if resolved:
        same_point = (lo_a == hi_a) & (lo_b == hi_b) & (lo_a == lo_b)
        amb &= ~same_point
    return amb


def _onehot(idx: torch.Tensor, R: int) -> torch.Tensor:
    """idx [..., k] -> bool [..., R]."""
    out = torch.zeros(*idx.shape[:-1], R, dtype=torch.bool)
    return out.scatter_(-1, idx, True)


def _pooled_bounds(lo, hi, req_mask):
    """Interval of amax over requesting rows: lo/hi [B,H,C,R], req_mask [B,H,C,R] -> [B,H,R]."""
    NEGd = torch.tensor(NEG, dtype=torch.float64)
    plo = torch.where(req_mask, lo, NEGd).max(dim=2).values
    phi = torch.where(req_mask, hi, NEGd).max(dim=2).values
    return plo, phi


# ---------------------------------------------------------------------------------------------
# prefill routing (one query chunk at a time)
# ---------------------------------------------------------------------------------------------
def _windows(p: OracleParams, n: int):
    """(f_hi, l_lo) for query chunk n (vectorized.py:242-253)."""
    kf, kl = max(0, p.keep_first), max(0, p.keep_last)
    f_hi = min(n, kf) if kf > 0 else 0
    l_lo = min(max(n - kl, kf), n) if kl > 0 else n
    return f_hi, l_lo


def _rank_topk(scores: torch.Tensor, k: int, sorted_: bool, rule: str = "torch"):
    """Top-k along the last axis.  ``rule="torch"``: ``torch.topk`` (the reference's call; its
    order among EQUAL scores is implementation-defined).  ``rule="index"``: the CUDA kernels' rule,
    higher score first and, among equal scores, the lower index; the result is then sorted by it."""
    R = scores.shape[-1]
    if k >= R:
        idx = torch.arange(R).expand(*scores.shape[:-1], R)
        return scores, idx, True
    if rule == "index":
        s, i = torch.sort(scores, dim=-1, descending=True, stable=True)
        return s[..., :k], i[..., :k], False
    s, i = torch.topk(scores, k, dim=-1, sorted=sorted_)
    return s, i, False


def _lowest_last(top_s: torch.Tensor, top_i: torch.Tensor) -> torch.Tensor:
    """Position in a top list of its lowest score, among equal lowest scores the highest index
    (the entry the kernels drop for the previous chunk); [..., 1]."""
    low = top_s == top_s.min(dim=-1, keepdim=True).values
    return torch.where(low, top_i, torch.full_like(top_i, -1)).argmax(dim=-1, keepdim=True)


def route_prefill(p: OracleParams, q: torch.Tensor, chunk_k: torch.Tensor, group_k: torch.Tensor,
                  S: int, chunks=None, ties: bool = True, acc_bound: float = _ACC_BOUND,
                  tie_rule: str = "torch") -> Dict[str, torch.Tensor]:
    """Two-level routing of the chunk-parallel prefill path, per query chunk.

    q ``[B,H,S,Dh]`` (RoPE applied); chunk_k ``[B,KVH,N,Dh]``; group_k ``[B,KVH,N,M,Dh]``.
    Returns per (b, h, n): ``chunk_idx``/``chunk_t0`` [.., Kc] and ``group_chunk``/
    ``group_idx``/``group_t0`` [.., Kg] in the reference's slot order, plus ``tie`` [B,H,N]
    flagging tiles whose selection depends on a near tie (see ``score_bounds``).  ``chunks``
    restricts the query chunks computed (others stay "never visible").  ``acc_bound`` is passed to
    ``score_bounds``.  ``tie_rule`` picks the order among equal scores (``_rank_topk``): ``"torch"``
    is the reference's, ``"index"`` the CUDA kernels'; under ``"index"`` the previous chunk
    replaces the lowest chosen chunk with the highest index, level-2 candidates are numbered in
    ascending chunk order, and the tie flags ignore equal scores (both sides order them alike).
    """
    rz = tie_rule == "index"
    B, H, _, Dh = q.shape
    C, M = p.chunk_size, p.M
    N = (S + C - 1) // C
    dtype = q.dtype
    rep = p.rep
    ck = chunk_k.repeat_interleave(rep, dim=1)                      # [B,H,N,Dh]
    gk = group_k.repeat_interleave(rep, dim=1)                      # [B,H,N,M,Dh]
    Kc = min(p.topk_chunks, N) if p.topk_chunks > 0 else 0
    Tgrp = Kc * M
    Kg = min(p.topk_groups, Tgrp) if p.topk_groups > 0 else 0
    Kgr = min(p.topk_groups // 2, Tgrp) if p.topk_groups > 0 else 0
    if Kg == 0 or Kgr == 0:
        Kg = 0
    out = {
        "chunk_idx": torch.full((B, H, N, Kc), -1, dtype=torch.long),
        "chunk_t0": torch.full((B, H, N, Kc), C, dtype=torch.long),
        "group_chunk": torch.full((B, H, N, Kg), -1, dtype=torch.long),
        "group_idx": torch.full((B, H, N, Kg), -1, dtype=torch.long),
        "group_t0": torch.full((B, H, N, Kg), C, dtype=torch.long),
        "tie": torch.zeros(B, H, N, dtype=torch.bool),
    }
    if Kc == 0:
        return out
    pad = N * C - S
    if pad:
        q = torch.cat([q, q.new_zeros(B, H, pad, Dh)], dim=2)
    cand = torch.arange(N)
    for n in (range(N) if chunks is None else chunks):
        f_hi, l_lo = _windows(p, n)
        qn = q[:, :, n * C:(n + 1) * C]                                  # [B,H,C,Dh]
        qvalid = (n * C + torch.arange(C)) < S                           # [C]
        pool = (cand < n) & (cand >= f_hi) & (cand < l_lo)               # [N]
        sc = torch.einsum("bhcd,bhmd->bhcm", qn, ck) * p.scale           # [B,H,C,N]
        rmask = pool.view(1, 1, 1, N) & qvalid.view(1, 1, C, 1)
        sc = sc.masked_fill(~rmask, NEG)
        req_s, req_i, all_req = _rank_topk(sc, Kc, sorted_=True, rule=tie_rule)
        if all_req:
            pooled = req_s.max(dim=-2).values                           # [B,H,N]
        else:
            pooled = torch.full((B * H, N), NEG, dtype=sc.dtype)
            pooled.scatter_reduce_(1, req_i.reshape(B * H, -1), req_s.reshape(B * H, -1),
                                   reduce="amax", include_self=True)
            pooled = pooled.view(B, H, N)
        top_s, top_i, _ = _rank_topk(pooled, Kc, sorted_=False, rule=tie_rule)
        tie = torch.zeros(B, H, dtype=torch.bool)
        if ties:
            lo, hi = score_bounds(qn, ck, p.scale, dtype, "bhcd,bhmd->bhcm", acc_bound)
            real = rmask.expand(B, H, C, N)
            req_m = _onehot(req_i, N) & real
            if not all_req:
                tie |= (_set_tie(lo, hi, req_m, real, rz) & qvalid.view(1, 1, C)).any(-1)
            if Kc < N:
                plo, phi = _pooled_bounds(lo, hi, req_m)
                preal = req_m.any(dim=2)
                tie |= _set_tie(plo, phi, _onehot(top_i, N), preal, rz)
        prev = n - 1
        if n > 0 and f_hi <= prev < l_lo:
            missing = ~(top_i == prev).any(dim=-1, keepdim=True)
            at = _lowest_last(top_s, top_i) if rz else top_s.argmin(dim=-1, keepdim=True)
            if ties and Kc < N:
                rem_i = top_i.gather(-1, at)                                 # [B,H,1]
                others = _onehot(top_i, N) & preal
                others.scatter_(-1, rem_i, False)
                amb = _pair_ambiguous(plo, phi, plo.gather(-1, rem_i), phi.gather(-1, rem_i), rz) & others
                tie |= missing.squeeze(-1) & amb.any(-1)
            top_i = top_i.scatter(-1, at, torch.where(missing, torch.full_like(at, prev),
                                                       top_i.gather(-1, at)))
        if rz:
            # the kernels number the level-2 candidates by ascending chunk id (their tie order)
            top_i = top_i.sort(dim=-1).values
        valid_prev = pool[top_i]                                         # [B,H,Kc]
        requested = (req_i.unsqueeze(-1) == top_i.view(B, H, 1, 1, Kc)).any(dim=-2)   # [B,H,C,Kc]
        requested &= valid_prev.unsqueeze(2)
        vis = (torch.cumsum(requested.int(), dim=2) > 0) & valid_prev.unsqueeze(2) & qvalid.view(1, 1, C, 1)
        if n > 0:
            vis |= (top_i == prev).unsqueeze(2) & qvalid.view(1, 1, C, 1)
        vis &= valid_prev.unsqueeze(2)
        out["chunk_idx"][:, :, n] = top_i
        out["chunk_t0"][:, :, n] = _first_true(vis, C)

        if Kg > 0:
            bidx = torch.arange(B).view(B, 1, 1)
            hidx = torch.arange(H).view(1, H, 1)
            cand_k = gk[bidx, hidx, top_i].reshape(B, H, Tgrp, Dh)        # [B,H,Kc*M,Dh]
            gvalid = valid_prev.unsqueeze(-1).expand(B, H, Kc, M).reshape(B, H, Tgrp)
            gsc = torch.einsum("bhcd,bhrd->bhcr", qn, cand_k) * p.scale      # [B,H,C,Tgrp]
            gmask = vis.unsqueeze(-1).expand(B, H, C, Kc, M).reshape(B, H, C, Tgrp)
            gmask = gmask & gvalid.unsqueeze(2) & qvalid.view(1, 1, C, 1)
            gsc = gsc.masked_fill(~gmask, NEG)
            greq_s, greq_i, gall = _rank_topk(gsc, Kgr, sorted_=True, rule=tie_rule)
            if gall:
                gpooled = greq_s.max(dim=-2).values
            else:
                gpooled = torch.full((B * H, Tgrp), NEG, dtype=gsc.dtype)
                gpooled.scatter_reduce_(1, greq_i.reshape(B * H, -1), greq_s.reshape(B * H, -1),
                                        reduce="amax", include_self=True)
                gpooled = gpooled.view(B, H, Tgrp)
            _, top_g, _ = _rank_topk(gpooled, Kg, sorted_=False, rule=tie_rule)
            if ties:
                glo, ghi = score_bounds(qn, cand_k, p.scale, dtype, "bhcd,bhrd->bhcr", acc_bound)
                greq_m = _onehot(greq_i, Tgrp) & gmask
                if not gall:
                    tie |= (_set_tie(glo, ghi, greq_m, gmask, rz) & qvalid.view(1, 1, C)).any(-1)
                if Kg < Tgrp:
                    gplo, gphi = _pooled_bounds(glo, ghi, greq_m)
                    tie |= _set_tie(gplo, gphi, _onehot(top_g, Tgrp), greq_m.any(dim=2), rz)
            top_gvalid = gvalid.gather(-1, top_g)
            parent = top_g // M
            parent_vis = vis.gather(-1, parent.unsqueeze(2).expand(B, H, C, Kg))
            greq = (greq_i.unsqueeze(-1) == top_g.view(B, H, 1, 1, Kg)).any(dim=-2)
            greq = greq & top_gvalid.unsqueeze(2) & parent_vis
            gvis = (torch.cumsum(greq.int(), dim=2) > 0) & top_gvalid.unsqueeze(2) & parent_vis
            gvis &= qvalid.view(1, 1, C, 1)
            out["group_chunk"][:, :, n] = top_i.gather(-1, parent)
            out["group_idx"][:, :, n] = top_g - parent * M
            out["group_t0"][:, :, n] = _first_true(gvis, C)
        out["tie"][:, :, n] = tie
    return out


def _first_true(vis: torch.Tensor, C: int) -> torch.Tensor:
    """vis [B,H,C,K] (monotone in the C axis over valid rows) -> first row index, C if none."""
    any_ = vis.any(dim=2)
    first = vis.int().argmax(dim=2)
    return torch.where(any_, first, torch.full_like(first, C))


def visible_sets(route: Dict[str, torch.Tensor], C: int, M: int):
    """Canonical per-(b,h,n) routing result: {abs group id: t0} and {chunk: t0}, visible only."""
    B, H, N = route["tie"].shape
    out = {}
    gc, gi, gt = route["group_chunk"], route["group_idx"], route["group_t0"]
    cc, ct = route["chunk_idx"], route["chunk_t0"]
    for b in range(B):
        for h in range(H):
            for n in range(N):
                g = {int(gc[b, h, n, j]) * M + int(gi[b, h, n, j]): int(gt[b, h, n, j])
                     for j in range(gc.shape[-1]) if int(gt[b, h, n, j]) < C}
                c = {int(cc[b, h, n, j]): int(ct[b, h, n, j])
                     for j in range(cc.shape[-1]) if int(ct[b, h, n, j]) < C}
                out[(b, h, n)] = (c, g)
    return out


# ---------------------------------------------------------------------------------------------
# prefill attention (one query chunk at a time)
# ---------------------------------------------------------------------------------------------
def attend_prefill(p: OracleParams, q, k_rope, v, route, S: int, chunks=None) -> torch.Tensor:
    """Token-only attention over the assembled working set, chunk_router.py:149-158.

    Key segments per query chunk n (vectorized.py:404-490): current chunk (causal), opened
    groups (row t sees group j iff t >= t0), last window [l_lo, n), first window [0, f_hi).
    Scores in fp32, masked_fill(NEG), fp32 softmax, fp32 P.V, cast to the value dtype.
    """
    B, H, _, Dh = q.shape
    C, gs = p.chunk_size, p.group_size
    N = (S + C - 1) // C
    rep = p.rep
    out = torch.zeros(B, H, S, Dh, dtype=v.dtype)
    kv_of_h = torch.arange(H) // rep
    Kg = route["group_t0"].shape[-1]
    for n in (range(N) if chunks is None else chunks):
        f_hi, l_lo = _windows(p, n)
        lo, hi = n * C, min(S, (n + 1) * C)
        L = hi - lo
        qn = q[:, :, lo:hi].float()                                        # [B,H,L,Dh]
        pos = [torch.arange(lo, hi).view(1, 1, L).expand(B, H, L)]
        msk = [(torch.arange(L).view(1, 1, 1, L) <= torch.arange(L).view(1, 1, L, 1)).expand(B, H, L, L)]
        if Kg:
            gpos = (route["group_chunk"][:, :, n] * C + route["group_idx"][:, :, n] * gs)
            gpos = gpos.clamp_min(0)
            tpos = (gpos.unsqueeze(-1) + torch.arange(gs)).reshape(B, H, Kg * gs).clamp_max(S - 1)
            t0 = route["group_t0"][:, :, n].unsqueeze(-1).expand(B, H, Kg, gs).reshape(B, H, Kg * gs)
            pos.append(tpos)
            msk.append(torch.arange(L).view(1, 1, L, 1) >= t0.unsqueeze(2))
        for a, b_ in ((l_lo, n), (0, f_hi)):
            if b_ > a:
                w = torch.arange(a * C, b_ * C)
                pos.append(w.view(1, 1, -1).expand(B, H, -1))
                msk.append(torch.ones(B, H, L, w.numel(), dtype=torch.bool))
        pos = torch.cat(pos, dim=2)                                        # [B,H,R]
        msk = torch.cat(msk, dim=3)                                        # [B,H,L,R]
        bi = torch.arange(B).view(B, 1, 1)
        ki = kv_of_h.view(1, H, 1)
        kk = k_rope[bi, ki, pos].float()                                   # [B,H,R,Dh]
        vv = v[bi, ki, pos].float()
        s = torch.einsum("bhld,bhrd->bhlr", qn, kk) * p.scale
        s = s.masked_fill(~msk, NEG)
        pr = torch.softmax(s, dim=-1)
        out[:, :, lo:hi] = torch.einsum("bhlr,bhrd->bhld", pr, vv).to(v.dtype)
    return out


# ---------------------------------------------------------------------------------------------
# decode (single active chunk, incremental path)
# ---------------------------------------------------------------------------------------------
def route_decode(p: OracleParams, q, chunk_k_mid, group_k_of, mid_lo: int, n_closed: int,
                 acc_bound: float = _ACC_BOUND, tie_rule: str = "torch"):
    """Routing of one decode block (chunk_router.py:188-277).

    q ``[B,H,L,Dh]``; chunk_k_mid ``[B,KVH,n_mid,Dh]`` = store chunk summaries of the routed
    pool; ``group_k_of(mid_idx[B,H,Kc]) -> [B,H,Kc,M,Dh]``.  Returns absolute chunk ids and
    group picks with their per-row first-visible index (L = never), plus a near-tie flag [B,H]
    (a selection that an accumulation-order difference of one rounding could flip; see
    ``score_bounds``).  ``acc_bound`` / ``tie_rule`` as in ``route_prefill``.
    """
    B, H, L, Dh = q.shape
    M = p.M
    rz = tie_rule == "index"
    dtype = q.dtype
    n_mid = chunk_k_mid.shape[2]
    ck = chunk_k_mid.repeat_interleave(p.rep, dim=1)
    res = {"mid_idx": torch.empty(B, H, 0, dtype=torch.long), "mid_t0": torch.empty(B, H, 0, dtype=torch.long),
           "open_chunk": torch.empty(B, H, 0, dtype=torch.long), "open_grp": torch.empty(B, H, 0, dtype=torch.long),
           "open_t0": torch.empty(B, H, 0, dtype=torch.long), "tie": torch.zeros(B, H, dtype=torch.bool)}
    if n_mid == 0 or p.topk_chunks <= 0:
        return res
    # chunk_router.py:222-232: scores in the model dtype, pooled by max over the block's rows
    sc = torch.einsum("bhld,bhnd->bhln", q, ck) * p.scale
    lo, hi = score_bounds(q, ck, p.scale, dtype, "bhld,bhnd->bhln", acc_bound)
    Kc = min(p.topk_chunks, n_mid)
    pooled = sc.max(dim=2).values
    top_s, mid_rel, _ = _rank_topk(pooled, Kc, False, tie_rule)
    _, req_rel, _ = _rank_topk(sc, Kc, False, tie_rule)
    plo, phi = lo.max(dim=2).values, hi.max(dim=2).values
    every = torch.ones_like(pooled, dtype=torch.bool)
    tie = _set_tie(plo, phi, _onehot(mid_rel, n_mid), every, rz)
    tie |= _set_tie(lo, hi, _onehot(req_rel, n_mid), torch.ones_like(sc, dtype=torch.bool), rz).any(-1)
    # chunk_router.py:234-246: the previous chunk replaces the lowest pooled pick
    prev = n_closed - 1
    mid_hi = mid_lo + n_mid
    prev_in = mid_lo <= prev < mid_hi
    if prev_in:
        prev_rel = prev - mid_lo
        missing = ~(mid_rel == prev_rel).any(dim=-1, keepdim=True)
        at = _lowest_last(top_s, mid_rel) if rz else top_s.argmin(dim=-1, keepdim=True)
        sel_lo, sel_hi = plo.gather(-1, mid_rel), phi.gather(-1, mid_rel)
        others = torch.ones_like(sel_lo, dtype=torch.bool).scatter(-1, at, False)
        amb = (_pair_ambiguous(sel_lo, sel_hi, sel_lo.gather(-1, at), sel_hi.gather(-1, at), rz)
               & others).any(-1, keepdim=True)
        tie |= (missing & amb).squeeze(-1)
        mid_rel = mid_rel.scatter(-1, at, torch.where(missing, torch.full_like(at, prev_rel), mid_rel.gather(-1, at)))
    if rz:
        mid_rel = mid_rel.sort(dim=-1).values    # level-2 candidates in ascending chunk order
    mid_idx = mid_rel + mid_lo
    mreq = (req_rel.unsqueeze(-2) == mid_rel.unsqueeze(2).unsqueeze(-1)).any(dim=-1)
    mvis = torch.cumsum(mreq.int(), dim=2) > 0
    if prev_in:
        mvis = mvis | (mid_rel == prev_rel).unsqueeze(2)
    res["mid_idx"], res["mid_t0"] = mid_idx, _first_true(mvis, L)
    Kg = min(p.topk_groups, Kc * M) if p.topk_groups > 0 else 0
    Kgr = min(p.topk_groups // 2, Kc * M) if p.topk_groups > 0 else 0
    if Kg <= 0:
        res["tie"] = tie
        return res
    # chunk_router.py:248-277: group candidates of the chosen chunks (not masked), pooled over rows
    gk = group_k_of(mid_idx).reshape(B, H, Kc * M, Dh)
    sg = torch.einsum("bhld,bhrd->bhlr", q, gk) * p.scale
    glo, ghi = score_bounds(q, gk, p.scale, dtype, "bhld,bhrd->bhlr", acc_bound)
    pg = sg.max(dim=2).values
    _, top_g, _ = _rank_topk(pg, Kg, False, tie_rule)
    tie |= _set_tie(glo.max(dim=2).values, ghi.max(dim=2).values, _onehot(top_g, Kc * M),
                    torch.ones_like(pg, dtype=torch.bool), rz)
    if Kgr > 0:
        _, req_g, _ = _rank_topk(sg, Kgr, False, tie_rule)
        tie |= _set_tie(glo, ghi, _onehot(req_g, Kc * M), torch.ones_like(sg, dtype=torch.bool), rz).any(-1)
        greq = (req_g.unsqueeze(-2) == top_g.unsqueeze(2).unsqueeze(-1)).any(dim=-1)
    else:
        greq = torch.zeros(B, H, L, Kg, dtype=torch.bool)
    parent = top_g // M
    ovis = (torch.cumsum(greq.int(), dim=2) > 0) & torch.gather(mvis, -1, parent.unsqueeze(2).expand(B, H, L, Kg))
    res["open_chunk"] = mid_idx.gather(-1, parent)
    res["open_grp"] = top_g - parent * M
    res["open_t0"] = _first_true(ovis, L)
    res["tie"] = tie
    return res


def attend_decode(p: OracleParams, q, keys, vals, key_first_row):
    """Flat attention of one decode block (chunk_router.py:159-162).

    keys/vals ``[B,H,R,Dh]`` (token keys of every segment), ``key_first_row`` [B,H,R]: the
    first query row (of L) that sees the key (L = never; causal current-chunk keys carry their
    own offset).  Returns ``[B,H,L,Dh]`` in the value dtype.
    """
    B, H, L, Dh = q.shape
    s = torch.einsum("bhld,bhrd->bhlr", q.float(), keys.float()) * p.scale
    msk = torch.arange(L).view(1, 1, L, 1) >= key_first_row.unsqueeze(2)
    s = s.masked_fill(~msk, NEG)
    return torch.einsum("bhlr,bhrd->bhld", torch.softmax(s, -1), vals.float()).to(vals.dtype)


def decode_sequence(p: OracleParams, q, k_rope, k_raw, v, block: int, start_pos: int = 0, calls=None,
                    attend=None, acc_bound: float = _ACC_BOUND, tie_rule: str = "torch"):
    """The reference's incremental path over a whole sequence: ``ChunkRouter.decode_block`` fed
    block by block and chunk-aligned (chunk_router.py:279-442), token-only attention.

    q ``[B,H,S,Dh]``, k_* / v ``[B,KVH,S,Dh]`` cover positions [0, S); rows before ``start_pos``
    are the already-closed prefix (its chunks are summarised exactly like closed decode chunks).
    ``calls`` (default ``[(start_pos, S)]``) are the caller's forward calls: each is fed in pieces
    of at most ``block`` tokens that never cross a chunk boundary (route_query_block,
    chunk_router.py:500-516).  ``attend(pos, L, rows, first)`` replaces the flat token attention
    (rows ``[B,H,R]`` absolute key positions, first ``[B,H,R]`` the first query row seeing each).
    Returns (out ``[B,H,S-start_pos,Dh]``, list of per-block dicts with ``pos``, ``L``, the
    routing result and its tie flag).
    """
    B, H, S, Dh = q.shape
    C, gs, rep = p.chunk_size, p.group_size, p.rep
    ck_all, gk_all, _ = summaries_store(p, k_raw, k_rope, v)
    kv_of_h = torch.arange(H) // rep
    bi = torch.arange(B).view(B, 1, 1)
    hi_ = kv_of_h.view(1, H, 1)
    if attend is None:
        def attend(pos, L, rows_t, first_t):
            return attend_decode(p, q[:, :, pos:pos + L], k_rope[bi, hi_, rows_t], v[bi, hi_, rows_t], first_t)
    outs, blocks = [], []
    for lo, hi in (calls if calls is not None else [(start_pos, S)]):
        pos = lo
        while pos < hi:
            L = min(block, C - pos % C, hi - pos)
            n, c0 = pos // C, pos % C
            f_hi, l_lo = _windows(p, n)
            qb = q[:, :, pos:pos + L]
            r = route_decode(p, qb, ck_all[:, :, f_hi:max(l_lo, f_hi)],
                             lambda mid: gk_all[bi, hi_, mid], f_hi, n, acc_bound, tie_rule)
            rows, first = [], []
            win = list(range(0, f_hi * C)) + list(range(l_lo * C, n * C))
            if win:
                rows.append(torch.tensor(win).view(1, 1, -1).expand(B, H, -1))
                first.append(torch.zeros(B, H, len(win), dtype=torch.long))
            if r["open_chunk"].shape[-1]:
                base = (r["open_chunk"] * C + r["open_grp"] * gs).unsqueeze(-1) + torch.arange(gs)
                rows.append(base.reshape(B, H, -1))
                first.append(r["open_t0"].unsqueeze(-1).expand(*r["open_t0"].shape, gs).reshape(B, H, -1))
            act = torch.arange(n * C, n * C + c0 + L)
            rows.append(act.view(1, 1, -1).expand(B, H, -1))
            first.append((torch.arange(c0 + L) - c0).view(1, 1, -1).expand(B, H, -1))
            outs.append(attend(pos, L, torch.cat(rows, -1), torch.cat(first, -1)))
            blocks.append({"pos": pos, "L": L, "route": r})
            pos += L
    return torch.cat(outs, dim=2), blocks


# ---------------------------------------------------------------------------------------------
# Dual Chunk Attention (the Qwen3 wrapper's dca_chunk > 0 path)
# ---------------------------------------------------------------------------------------------
DCA_NEG = -1.0e4  # finite mask fill of the DCA attention (qwen_routed_attention.py:63)


def dca_rope_table(positions: torch.Tensor, head_dim: int, theta: float, dtype: torch.dtype):
    """Default-RoPE cos/sin ``[*positions.shape, Dh]`` at (remapped) positions, cast to ``dtype``
    (qwen_routed_attention.py:66-81)."""
    half = head_dim // 2
    inv = 1.0 / (theta ** (torch.arange(half, dtype=torch.float32) / half))
    f = positions.to(torch.float32).unsqueeze(-1) * inv
    emb = torch.cat((f, f), dim=-1)
    return emb.cos().to(dtype), emb.sin().to(dtype)


def dca_apply(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """rotate-half RoPE evaluated in x's dtype, each operation rounded like the reference's
    (qwen_routed_attention.py:84-88)."""
    half = x.shape[-1] // 2
    return x * cos + torch.cat((-x[..., half:], x[..., :half]), dim=-1) * sin


def dca_sequence(p: OracleParams, q_raw, k_raw, v, dca_chunk: int, dca_local: int, calls,
                 acc_bound: float = _ACC_BOUND, tie_rule: str = "torch"):
    """The wrapper's Dual Chunk Attention over a sequence fed as forward ``calls`` [(lo, hi)]
    (qwen_routed_attention.py:210-283).

    Keys are roped at their intra-chunk position ``pos % dca_chunk`` and routed with intra-roped
    queries through the incremental path (route_query_block with return_positions); each query
    then scores a key with one of three ropings of itself, chosen by the two DCA-chunk indices:
    intra (same chunk, position pos % L_c), successor (the chunk just before, min(pos % L_c + L_c,
    ceil)) or inter (any earlier chunk, ceil), ceil = dca_chunk + dca_local.  q_raw ``[B,H,S,Dh]``
    and k_raw / v ``[B,KVH,S,Dh]`` are pre-RoPE.  Returns (out ``[B,H,S,Dh]``, routing blocks).
    """
    B, H, S, Dh = q_raw.shape
    L_c, ceil = dca_chunk, dca_chunk + dca_local
    pos = torch.arange(S)
    c_, s_ = dca_rope_table(pos % L_c, Dh, p.theta, k_raw.dtype)
    k_dca = dca_apply(k_raw, c_, s_)
    q_sel = dca_apply(q_raw, c_, s_)
    bi = torch.arange(B).view(B, 1, 1)
    hi_ = (torch.arange(H) // p.rep).view(1, H, 1)

    def attend(pos0, L, rows_t, first_t):
        qf = q_raw[:, :, pos0:pos0 + L].float()
        qpos = torch.arange(pos0, pos0 + L)
        qp = qpos % L_c
        q_i = dca_apply(qf, *dca_rope_table(qp, Dh, p.theta, torch.float32))
        q_s = dca_apply(qf, *dca_rope_table((qp + L_c).clamp(max=ceil), Dh, p.theta, torch.float32))
        q_t = dca_apply(qf, *dca_rope_table(torch.full_like(qpos, ceil), Dh, p.theta, torch.float32))
        kf = k_dca[bi, hi_, rows_t].float()
        vals = v[bi, hi_, rows_t]
        s_i = torch.einsum("bhld,bhrd->bhlr", q_i, kf) * p.scale
        s_s = torch.einsum("bhld,bhrd->bhlr", q_s, kf) * p.scale
        s_t = torch.einsum("bhld,bhrd->bhlr", q_t, kf) * p.scale
        cq = (qpos // L_c).view(1, 1, L, 1)
        ck = (rows_t // L_c).unsqueeze(2)
        sc = torch.where(ck == cq, s_i, torch.where(ck == cq - 1, s_s, s_t))
        seen = torch.arange(L).view(1, 1, L, 1) >= first_t.unsqueeze(2)
        sc = sc.masked_fill(~seen, DCA_NEG)
        return torch.einsum("bhlr,bhrd->bhld", torch.softmax(sc, -1), vals.float()).to(vals.dtype)

    return decode_sequence(p, q_sel, k_dca, k_raw, v, p.chunk_size, calls=calls, attend=attend, acc_bound=acc_bound,
                           tie_rule=tie_rule)


# ---------------------------------------------------------------------------------------------
# module-level helpers (projection prologue of HierarchicalGlobalAttentionRouted.forward)
# ---------------------------------------------------------------------------------------------
def rms_norm(x: torch.Tensor, w: Optional[torch.Tensor], eps: float) -> torch.Tensor:
    """RMSNorm of the reference module (HierarchicalGlobalAttentionRouted.py:56-67)."""
    if w is None:
        return x
    xf = x.float()
    return (w.float() * xf * torch.rsqrt(xf.pow(2).mean(dim=-1, keepdim=True) + eps)).to(x.dtype)


def module_rotary(theta: float, head_dim: int, S: int, start: int = 0):
    """fp32 cos/sin ``[S, Dh]`` (HierarchicalGlobalAttentionRouted.py:209-217)."""
    half = head_dim // 2
    inv = 1.0 / (theta ** (torch.arange(0, half, dtype=torch.float32) / half))
    t = torch.arange(start + S, dtype=torch.float32)
    f = torch.einsum("i,j->ij", t, inv)
    emb = torch.cat((f, f), dim=-1)
    return emb.cos()[start:], emb.sin()[start:]


def module_forward(p: OracleParams, x, wq, wk, wv, wo, qn_w, kn_w, eps, chunks=None):
    """Prefill forward of the routed module at start_pos 0 (HierarchicalGlobalAttentionRouted.py:137-177).

    Returns (out [B,S,d_model], intermediates dict).  ``chunks`` restricts the routed query
    chunks (the CPU-baseline sample); the other rows of ``out`` are then meaningless.
    """
    B, S, _ = x.shape
    H, KVH, Dh = p.nhead, p.kv_heads, p.head_dim
    q_raw = rms_norm((x @ wq.t()).view(B, S, H, Dh), qn_w, eps).transpose(1, 2)
    k_raw = rms_norm((x @ wk.t()).view(B, S, KVH, Dh), kn_w, eps).transpose(1, 2)
    v = (x @ wv.t()).view(B, S, KVH, Dh).transpose(1, 2)
    cos, sin = module_rotary(p.theta, Dh, S)
    q_rope = _rotate(q_raw.float(), cos, sin).to(q_raw.dtype)
    k_rope = _rotate(k_raw.float(), cos, sin).to(k_raw.dtype)
    cos_r, sin_r = cos.to(x.dtype), sin.to(x.dtype)
    ck, gk, gv = summaries_prefill(p, k_raw.contiguous(), k_rope.contiguous(), v.contiguous(), cos_r, sin_r)
    route = route_prefill(p, q_rope, ck, gk, S, chunks=chunks)
    heads = attend_prefill(p, q_rope, k_rope, v, route, S, chunks=chunks)
    out = heads.transpose(1, 2).reshape(B, S, H * Dh) @ wo.t()
    return out, {"q_rope": q_rope, "k_rope": k_rope, "k_raw": k_raw, "v": v, "chunk_k": ck,
                 "group_k": gk, "group_v": gv, "route": route, "heads": heads}
