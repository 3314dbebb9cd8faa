"""Generate the golden fixtures by running the UNMODIFIED reference implementation.

Run here (where the reference checkout is readable):

    PYTHONDONTWRITEBYTECODE=1 python tests/golden/make_golden.py [--ref /path/to/reference]

Each case draws seeded inputs (``cases.make_inputs``), runs the reference's own code path
(``assemble_routed_kv`` + ``RoutedKV.attend`` for prefill, ``ChunkRouter.decode_block`` +
``attend`` for the incremental path, the ``HierarchicalGlobalAttentionRouted`` module for the
module case, the Qwen3 wrapper's Dual Chunk Attention methods for the DCA cases) and stores the outputs and routing decisions as ``tests/golden/<case>.pt``.
Routing decisions are captured by wrapping the reference's own gather helpers, which receive
the selected chunk / group indices (vectorized.py:339, 388) — the reference is not modified.
Large tensors (inputs) are NOT stored; they are regenerated from the seed and checked with a
stored checksum.  Outputs are stored on a row subset for the larger cases.
"""
from __future__ import annotations

import argparse
import os
import sys

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
import cases  # noqa: E402


def _import_reference(ref_root: str):
    sys.dont_write_bytecode = True
    eft = os.path.join(ref_root, "ExistingModelFineTuning")
    for p in (ref_root, eft):
        if p not in sys.path:
            sys.path.insert(0, p)
    import KvRouter.vectorized as vec  # type: ignore
    from KvRouter import ChunkRouter, RouterConfig, VramKVCacheStore, RamKVCacheStore  # type: ignore
    from KvRouter.cache_store import ChunkPlacementPolicy  # type: ignore
    import HierarchicalGlobalAttentionRouted as hgar  # type: ignore
    sys.path.insert(0, os.path.join(eft, "Qwen3LongContext"))
    import qwen_routed_attention as qra  # type: ignore
    hgar.__qwen__ = qra
    return vec, ChunkRouter, RouterConfig, VramKVCacheStore, RamKVCacheStore, ChunkPlacementPolicy, hgar


def _first_true(mask: torch.Tensor, C: int) -> torch.Tensor:
    any_ = mask.any(dim=-2)
    first = mask.int().argmax(dim=-2)
    return torch.where(any_, first, torch.full_like(first, C))


def run_prefill_case(ref, case):
    vec, ChunkRouter, RouterConfig, VramKVCacheStore, _, Policy, _ = ref
    p = case["params"]
    inp = cases.make_inputs(case)
    q, k_rope, k_raw, v, cos, sin = (inp[k] for k in ("q", "k_rope", "k_raw", "v", "cos", "sin"))
    B, H, S, Dh = q.shape
    C, gs = p.chunk_size, p.group_size
    M = C // gs
    cfg = RouterConfig(nhead=p.nhead, kv_heads=p.kv_heads, head_dim=Dh, chunk_size=C, group_size=gs,
                       topk_chunks=p.topk_chunks, topk_groups=p.topk_groups, theta=p.theta)
    policy = Policy(keep_first=p.keep_first, keep_last=p.keep_last, first_token_level=True)
    store = VramKVCacheStore(compute_device=torch.device("cpu"), policy=policy, kv_heads=p.kv_heads,
                             head_dim=Dh, chunk_size=C, groups_per_chunk=M, batch_size=B, dtype=q.dtype)
    router = ChunkRouter(cfg, store)

    captured = {}
    orig_gc, orig_gg = vec._gather_chunks, vec._gather_groups

    def gc(t, idx):
        captured.setdefault("top_chunk_idx", idx.clone())
        return orig_gc(t, idx)

    def gg(t, cidx, gidx):
        captured.setdefault("src_chunk", cidx.clone())
        captured.setdefault("src_group", gidx.clone())
        return orig_gg(t, cidx, gidx)

    vec._gather_chunks, vec._gather_groups = gc, gg
    try:
        segs = router.route_query_block(0, q, k_rope, k_raw, v, 0, cos=cos.view(1, 1, S, Dh),
                                        sin=sin.view(1, 1, S, Dh))
    finally:
        vec._gather_chunks, vec._gather_groups = orig_gc, orig_gg
    assert len(segs) == 1
    routed = segs[0][0]
    out = routed.attend(q, use_summaries=False)

    N = (S + C - 1) // C
    gold = {"name": case["name"], "input_checksum": cases.checksum(inp)}
    Kc = min(p.topk_chunks, N) if p.topk_chunks > 0 else 0
    Tgrp = Kc * M
    Kg = min(p.topk_groups, Tgrp) if p.topk_groups > 0 else 0
    Kgr = min(p.topk_groups // 2, Tgrp) if p.topk_groups > 0 else 0
    if Kc > 0:
        gold["chunk_idx"] = captured["top_chunk_idx"].to(torch.int32)
        # chunk visibility = group_summary_mask columns k*M (valid groups of complete chunks)
        sm = routed.summary_mask[..., :Tgrp].reshape(B, H, N, C, Kc, M)[..., 0]
        gold["chunk_t0"] = _first_true(sm, C).to(torch.int16)
    if Kg > 0 and Kgr > 0:
        gold["group_chunk"] = captured["src_chunk"].to(torch.int32)
        gold["group_idx"] = captured["src_group"].to(torch.int16)
        tm = routed.token_mask[..., C:C + Kg * gs].reshape(B, H, N, C, Kg, gs)[..., 0]
        gold["group_t0"] = _first_true(tm, C).to(torch.int16)
    rows = cases.output_rows(case, S)
    gold["out_rows"] = rows
    gold["out"] = out[:, :, rows].clone()
    return gold


def run_summary_case(ref, case):
    vec, _, RouterConfig, _, _, _, _ = ref
    p = case["params"]
    inp = cases.make_inputs(case)
    k_rope, k_raw, v, cos, sin = (inp[k] for k in ("k_rope", "k_raw", "v", "cos", "sin"))
    B, KVH, S, Dh = k_raw.shape
    C, gs = p.chunk_size, p.group_size
    M = C // gs
    cfg = RouterConfig(nhead=p.kv_heads, kv_heads=p.kv_heads, head_dim=Dh, chunk_size=C, group_size=gs,
                       theta=p.theta)
    N = (S + C - 1) // C
    Sp = N * C
    pad = Sp - S

    def padded(x):
        return torch.cat([x, x.new_zeros(B, KVH, pad, Dh)], dim=2) if pad else x

    valid = (torch.arange(Sp) < S).view(N, C)
    chunk_len = valid.sum(1)
    c_mid = (torch.arange(N) * C + (chunk_len.clamp_min(1) - 1) // 2).clamp_max(S - 1)
    g_len = valid.view(N, M, gs).sum(-1)
    g_start = torch.arange(N)[:, None] * C + torch.arange(M)[None, :] * gs
    g_mid = (g_start + (g_len.clamp_min(1) - 1) // 2).clamp_max(S - 1)
    raw = padded(k_raw).reshape(B, KVH, N, C, Dh)
    rope = padded(k_rope).reshape(B, KVH, N, C, Dh)
    cos4, sin4 = cos.view(1, 1, S, Dh), sin.view(1, 1, S, Dh)
    # the reference's own summary function, called exactly as vectorized.py:275-287 does
    ck = vec._rope_summary(cfg, raw, rope, valid.view(1, 1, N, C, 1).to(k_raw.dtype), 3, c_mid, cos4, sin4, 1.0)
    gk = vec._rope_summary(cfg, raw.reshape(B, KVH, N, M, gs, Dh), rope.reshape(B, KVH, N, M, gs, Dh),
                           valid.view(1, 1, N, M, gs, 1).to(k_raw.dtype), 4, g_mid, cos4, sin4,
                           cfg.group_kv_scale)
    return {"name": case["name"], "input_checksum": cases.checksum(inp), "chunk_k": ck, "group_k": gk}


def run_incremental_case(ref, case):
    """Reference incremental path: ChunkRouter.prefill (decode_block per chunk-aligned slice)."""
    _, ChunkRouter, RouterConfig, VramKVCacheStore, RamKVCacheStore, Policy, _ = ref
    p = case["params"]
    inp = cases.make_inputs(case)
    q, k_rope, k_raw, v = (inp[k] for k in ("q", "k_rope", "k_raw", "v"))
    B, H, S, Dh = q.shape
    C, gs = p.chunk_size, p.group_size
    cfg = RouterConfig(nhead=p.nhead, kv_heads=p.kv_heads, head_dim=Dh, chunk_size=C, group_size=gs,
                       topk_chunks=p.topk_chunks, topk_groups=p.topk_groups, theta=p.theta)
    policy = Policy(keep_first=p.keep_first, keep_last=p.keep_last, first_token_level=True)
    store = RamKVCacheStore(compute_device=torch.device("cpu"), policy=policy, kv_heads=p.kv_heads,
                            head_dim=Dh, chunk_size=C, groups_per_chunk=C // gs, batch_size=B,
                            dtype=q.dtype, pin_memory=False)
    router = ChunkRouter(cfg, store)
    blk = case.get("block", C)
    outs, pos = [], 0
    while pos < S:
        take = min(blk, C - (pos % C), S - pos)
        sl = slice(pos, pos + take)
        routed = router.decode_block(0, q[:, :, sl], k_rope[:, :, sl], k_raw[:, :, sl], v[:, :, sl], pos)
        outs.append(routed.attend(q[:, :, sl], use_summaries=False))
        pos += take
    out = torch.cat(outs, dim=2)
    rows = cases.output_rows(case, S)
    return {"name": case["name"], "input_checksum": cases.checksum(inp), "out_rows": rows,
            "out": out[:, :, rows].clone(),
            "store_chunk_k": store.chunk_summaries(0).clone()}


def run_module_case(ref, case):
    hgar = ref[-1]
    p = case["params"]
    inp = cases.make_module_inputs(case)
    m = hgar.HierarchicalGlobalAttentionRouted(
        d_model=inp["x"].shape[-1], nhead=p.nhead, kv_heads=p.kv_heads, head_dim=p.head_dim,
        chunk_size=p.chunk_size, group_size=p.group_size, topk_chunks=p.topk_chunks,
        topk_groups=p.topk_groups, keep_first=p.keep_first, keep_last=p.keep_last,
        qk_norm=case.get("qk_norm", False), theta=p.theta)
    cases.load_module_weights(m, inp)
    m = m.to(inp["x"].dtype)
    with torch.no_grad():
        out, _ = m(inp["x"])
    rows = cases.output_rows(case, inp["x"].shape[1])
    return {"name": case["name"], "input_checksum": cases.checksum(inp), "out_rows": rows,
            "out": out[:, rows].clone()}


def run_qwen_case(ref, case):
    """The reference's QwenRoutedAttention over HF Qwen3MoeAttention on the case's schedule."""
    import types
    from transformers.models.qwen3_moe.modeling_qwen3_moe import Qwen3MoeAttention, Qwen3MoeRotaryEmbedding
    qra = ref[-1].__qwen__
    p = case["params"]
    inp = cases.make_qwen_inputs(case)
    cfg = cases.qwen_config(case)
    attn = Qwen3MoeAttention(cfg, layer_idx=0).to(inp["x"].dtype).eval()
    cases.load_qwen_weights(attn, inp)
    rot = Qwen3MoeRotaryEmbedding(cfg)
    x = inp["x"]
    S = x.shape[1]
    pos = torch.arange(S).unsqueeze(0)
    cos, sin = rot(x, pos)
    w = qra.QwenRoutedAttention(attn, cfg, keep_first=p.keep_first, keep_last=p.keep_last,
                                topk_chunks=p.topk_chunks, topk_groups=p.topk_groups, chunk_size=p.chunk_size,
                                group_size=p.group_size)
    pkv = types.SimpleNamespace()
    outs = []
    with torch.no_grad():
        for lo, hi in cases.qwen_schedule(case):
            o, _ = w(x[:, lo:hi], position_embeddings=(cos[:, lo:hi], sin[:, lo:hi]), attention_mask=None,
                     past_key_values=pkv, position_ids=pos[:, lo:hi])
            outs.append(o)
    out = torch.cat(outs, dim=1)
    rows = cases.output_rows(case, S)
    return {"name": case["name"], "input_checksum": cases.checksum(inp), "out_rows": rows,
            "out": out[:, rows].clone()}


def run_dca_case(ref, case):
    """The reference wrapper's Dual Chunk Attention (QwenRoutedAttention._dca_forward and
    _dca_attend, qwen_routed_attention.py:210-283) over the case's call schedule.  The two methods
    read only the attributes set below, so they run on a plain namespace carrying them, with an
    identity o_proj (the output is then the concatenated heads)."""
    import types
    _, ChunkRouter, RouterConfig, VramKVCacheStore, _, Policy, hgar = ref
    qra = hgar.__qwen__
    p = case["params"]
    inp = cases.make_dca_inputs(case)
    q, k_raw, v = inp["q"], inp["k_raw"], inp["v"]
    B, H, S, Dh = q.shape
    C, gs = p.chunk_size, p.group_size
    cfg = RouterConfig(nhead=p.nhead, kv_heads=p.kv_heads, head_dim=Dh, chunk_size=C, group_size=gs,
                       topk_chunks=p.topk_chunks, topk_groups=p.topk_groups, theta=p.theta)
    policy = Policy(keep_first=p.keep_first, keep_last=p.keep_last, first_token_level=True)
    store = VramKVCacheStore(compute_device=torch.device("cpu"), policy=policy, kv_heads=p.kv_heads,
                             head_dim=Dh, chunk_size=C, groups_per_chunk=C // gs, batch_size=B, dtype=q.dtype)
    router = ChunkRouter(cfg, store)
    w = types.SimpleNamespace(num_heads=H, num_kv_heads=p.kv_heads, head_dim=Dh, layer_idx=0, _cfg=cfg,
                              dca_chunk=case["dca_chunk"], dca_ceil=case["dca_chunk"] + case["dca_local"])
    w._dca_attend = lambda qb, routed, qpos: qra.QwenRoutedAttention._dca_attend(w, qb, routed, qpos)
    o = types.SimpleNamespace(o_proj=lambda x: x)
    outs = []
    with torch.no_grad():
        for lo, hi in cases.qwen_schedule(case):
            y, _ = qra.QwenRoutedAttention._dca_forward(w, o, q[:, :, lo:hi], k_raw[:, :, lo:hi],
                                                        v[:, :, lo:hi], lo, router, B, hi - lo)
            outs.append(y.view(B, hi - lo, H, Dh).transpose(1, 2))
    out = torch.cat(outs, dim=2)
    rows = cases.output_rows(case, S)
    return {"name": case["name"], "input_checksum": cases.checksum(inp), "out_rows": rows,
            "out": out[:, :, rows].clone()}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("HGA_REFERENCE_ROOT"),
                    help="checkout of the reference repository (or set HGA_REFERENCE_ROOT)")
    ap.add_argument("--only", default=None)
    args = ap.parse_args()
    if not args.ref:
        ap.error("--ref (or HGA_REFERENCE_ROOT) must point at the reference checkout")
    ref = _import_reference(args.ref)
    torch.set_num_threads(os.cpu_count() or 1)
    for case in cases.CASES:
        if args.only and case["name"] != args.only:
            continue
        kind = case["kind"]
        fn = {"prefill": run_prefill_case, "summary": run_summary_case,
              "incremental": run_incremental_case, "module": run_module_case, "qwen": run_qwen_case,
              "dca": run_dca_case}[kind]
        gold = fn(ref, case)
        path = os.path.join(HERE, f"{case['name']}.pt")
        torch.save(gold, path)
        print(f"wrote {path} ({os.path.getsize(path) / 1024:.1f} KiB)")


if __name__ == "__main__":
    main()
