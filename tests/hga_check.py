"""Parity checkers shared by the GPU tests (CPU-side, test infrastructure only).

* ``replay_prefill_selection`` re-derives, from the routing scores the kernel itself dumped,
  what the reference's selection rules yield under the kernel's tie rule (higher score, then
  lower index) — an exact check of the kernel's selection logic.
* ``check_scores_in_bounds`` checks every dumped score lies in the oracle's possible-score
  interval (fp64 dot product widened by an fp32 accumulation bound, then the reference's
  rounding points).
* ``gpu_sets`` / ``compare_to_oracle`` compare visible chunk / group sets with the oracle (the
  reference's own torch.topk order) and require every mismatching tile to be a flagged near tie.
"""
from __future__ import annotations

import numpy as np
import torch

from oracle import hga_oracle as O


def _windows(p, n):
    return O._windows(p, n)


def sizes(p, S):
    C, M = p.chunk_size, p.M
    N = (S + C - 1) // C
    Kc = min(p.topk_chunks, N) if p.topk_chunks > 0 else 0
    Tg = Kc * M
    Kg = min(p.topk_groups, Tg) if p.topk_groups > 0 else 0
    Kgr = min(p.topk_groups // 2, Tg) if p.topk_groups > 0 else 0
    if Kgr == 0:
        Kg = 0
    return N, Kc, Kg, Kgr, Tg


def _top(vals, idxs, k):
    """top-k of (vals, idxs) by (-val, idx)."""
    order = sorted(range(len(idxs)), key=lambda i: (-vals[i], idxs[i]))
    return [idxs[i] for i in order[:k]]


def replay_prefill_selection(p, S, res, chunks=None, offset=0):
    """Returns the expected (sel_chunk, sel_t0, open_gid, open_t0) lists per tile from dumped scores.
    ``chunks`` (default all) are absolute query chunks; the dumps hold chunk n at index n - offset
    (a ``chunk_range`` call)."""
    C, M = p.chunk_size, p.M
    N, Kc, Kg, Kgr, Tg = sizes(p, S)
    l1 = res["dbg_l1"].cpu().numpy()
    l2 = res["dbg_l2"].cpu().numpy()
    B, H = l1.shape[:2]
    exp = {}
    for b in range(B):
        for h in range(H):
            for n in (range(N) if chunks is None else chunks):
                ln = n - offset
                sel, open_ = [], []
                f_hi, l_lo = _windows(p, n)
                pool = list(range(f_hi, l_lo))
                nvalid = min(C, S - n * C)
                if Kc and pool:
                    k1 = min(Kc, len(pool))
                    pooled, t0 = {}, {}
                    for t in range(nvalid):
                        row = [float(l1[b, h, ln, t, c]) for c in pool]
                        for c in _top(row, pool, k1):
                            pooled[c] = max(pooled.get(c, -np.inf), float(l1[b, h, ln, t, c]))
                            t0.setdefault(c, t)
                    req = sorted(pooled)
                    chosen = req if len(req) <= Kc else _top([pooled[c] for c in req], req, Kc)
                    chosen = set(chosen)
                    prev = n - 1
                    if n > 0 and f_hi <= prev < l_lo:
                        if prev not in chosen:
                            if len(chosen) >= Kc:
                                worst = sorted(chosen, key=lambda c: (pooled[c], -c))[0]
                                chosen.discard(worst)
                            chosen.add(prev)
                        t0[prev] = 0
                    sel = [(c, t0[c]) for c in sorted(chosen)]
                    if Kg:
                        tsel = len(sel) * M
                        gpool, gt0 = {}, {}
                        for t in range(nvalid):
                            real = [j for j in range(tsel) if t >= sel[j // M][1]]
                            vals = [float(l2[b, h, ln, t, j]) for j in real]
                            reqj = real if Kgr >= Tg else _top(vals, real, Kgr)
                            for j in reqj:
                                gpool[j] = max(gpool.get(j, -np.inf), float(l2[b, h, ln, t, j]))
                                gt0.setdefault(j, t)
                        js = sorted(gpool)
                        if Kg < Tg and len(js) > Kg:
                            js = sorted(_top([gpool[j] for j in js], js, Kg))
                        open_ = [(sel[j // M][0] * M + j % M, gt0[j]) for j in js]
                exp[(b, h, n)] = (sel, open_)
    return exp


def gpu_lists(res, key_a, key_b, offset=0, chunks=None):
    """{(b, h, n): [(id, t0), ...]} of a GPU routing result whose index n - offset holds chunk n."""
    a = res[key_a].cpu().numpy()
    bb = res[key_b].cpu().numpy()
    out = {}
    B, H, N = a.shape[:3]
    for b in range(B):
        for h in range(H):
            for n in (range(offset, offset + N) if chunks is None else chunks):
                ln = n - offset
                out[(b, h, n)] = [(int(x), int(y)) for x, y in zip(a[b, h, ln], bb[b, h, ln]) if x >= 0]
    return out


def check_replay(p, S, res, chunks=None, offset=0):
    exp = replay_prefill_selection(p, S, res, chunks, offset)
    sel = gpu_lists(res, "sel_chunk", "sel_t0", offset, chunks)
    opn = gpu_lists(res, "open_gid", "open_t0", offset, chunks)
    bad = [k for k in exp if exp[k][0] != sel[k] or exp[k][1] != opn[k]]
    return bad, exp


def check_scores_in_bounds(p, S, q, chunk_k, group_k, res, chunks=None, offset=0):
    """Every dumped (valid, real) score lies in the oracle's possible-score interval.  ``chunks`` /
    ``offset`` as in ``replay_prefill_selection`` (q always holds the whole sequence)."""
    C, M = p.chunk_size, p.M
    N, Kc, Kg, Kgr, Tg = sizes(p, S)
    dtype = q.dtype
    qc = q.cpu()
    ck = chunk_k.cpu().repeat_interleave(p.rep, dim=1)
    gk = group_k.cpu().repeat_interleave(p.rep, dim=1)
    l1 = res["dbg_l1"].cpu()
    l2 = res["dbg_l2"].cpu()
    sel = res["sel_chunk"].cpu()
    B, H = qc.shape[:2]
    worst = 0
    for n in (range(N) if chunks is None else chunks):
        ln = n - offset
        f_hi, l_lo = _windows(p, n)
        nvalid = min(C, S - n * C)
        qn = qc[:, :, n * C:n * C + nvalid]
        if l_lo > f_hi and Kc:
            lo, hi = O.score_bounds(qn, ck[:, :, f_hi:l_lo], p.scale, dtype, "bhcd,bhmd->bhcm")
            got = l1[:, :, ln, :nvalid, f_hi:l_lo].double()
            worst = max(worst, int(((got < lo) | (got > hi)).sum()))
        if Kg:
            s = sel[:, :, ln]
            ksel = int((s[0, 0] >= 0).sum()) if s.numel() else 0
            for b in range(B):
                for h in range(H):
                    cs = [int(x) for x in s[b, h] if x >= 0]
                    if not cs:
                        continue
                    keys = gk[b, h, cs].reshape(len(cs) * M, -1)
                    lo, hi = O.score_bounds(qn[b, h], keys, p.scale, dtype, "cd,rd->cr")
                    got = l2[b, h, ln, :nvalid, :len(cs) * M].double()
                    real = got > O.NEG
                    worst = max(worst, int((((got < lo) | (got > hi)) & real).sum()))
            del ksel
    return worst


def oracle_sets(route, C, M):
    return O.visible_sets(route, C, M)


def gpu_sets(res, M, chunks=None, offset=0):
    sel = gpu_lists(res, "sel_chunk", "sel_t0", offset, chunks)
    opn = gpu_lists(res, "open_gid", "open_t0", offset, chunks)
    return {k: (dict(sel[k]), dict(opn[k])) for k in sel}


def oracle_sets_for(route, C, M, chunks):
    """``oracle_sets`` restricted to the query chunks ``chunks`` (long sequences)."""
    B, H, _ = route["tie"].shape
    gc, gi, gt = (route[k].numpy() for k in ("group_chunk", "group_idx", "group_t0"))
    cc, ct = route["chunk_idx"].numpy(), route["chunk_t0"].numpy()
    out = {}
    for b in range(B):
        for h in range(H):
            for n in chunks:
                g = {int(x) * M + int(y): int(t) for x, y, t in zip(gc[b, h, n], gi[b, h, n], gt[b, h, n]) if t < C}
                c = {int(x): int(t) for x, t in zip(cc[b, h, n], ct[b, h, n]) if t < C}
                out[(b, h, n)] = (c, g)
    return out


def tie_report(osets, gsets, tie):
    """Compare visible sets tile by tile; ``tie`` [B,H,N] are the oracle's near-tie flags.  Returns
    the tile count, the mismatching tiles, those NOT flagged, the flagged share and the mean
    Jaccard similarity of the opened-group sets over the mismatching tiles."""
    keys = sorted(osets)
    mism = [k for k in keys if osets[k] != gsets[k]]
    unexplained = [k for k in mism if not bool(tie[k])]
    jac = []
    for k in mism:
        a, b = set(osets[k][1]), set(gsets[k][1])
        jac.append(len(a & b) / max(1, len(a | b)))
    n = max(1, len(keys))
    return {"tiles": len(keys), "mismatch": len(mism), "unexplained": unexplained,
            "tie_frac": sum(bool(tie[k]) for k in keys) / n, "mismatch_frac": len(mism) / n,
            "mismatch_jaccard": (sum(jac) / len(jac)) if jac else 1.0}


def route_dict_from_gpu(res, p, S):
    """GPU open lists in the oracle's route-dict form (for oracle attention on GPU routing)."""
    C, M = p.chunk_size, p.M
    gid = res["open_gid"].cpu().long()
    t0 = res["open_t0"].cpu().long()
    valid = gid >= 0
    return {"group_chunk": torch.where(valid, gid // M, torch.full_like(gid, -1)),
            "group_idx": torch.where(valid, gid % M, torch.full_like(gid, -1)),
            "group_t0": torch.where(valid, t0, torch.full_like(t0, C)),
            "tie": torch.zeros(gid.shape[:3], dtype=torch.bool)}


def attn_errors(out, ref, dtype):
    """(max-abs, mean-relative) errors of an attention output vs its reference."""
    d = (out.float() - ref.float()).abs()
    mean_rel = (d.sum() / ref.float().abs().sum().clamp_min(1e-30)).item()
    return d.max().item(), mean_rel


TOL = {torch.bfloat16: (2e-2, 5e-3), torch.float16: (2e-2, 5e-3), torch.float32: (1e-4, 1e-5)}
