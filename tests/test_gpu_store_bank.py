"""The RAM tier's VRAM token bank (hga_gather_h2d): the counterpart of the reference's bank tests
(ExistingModelFineTuning/KvRouter/Tests/test_summary_cache.py:47-119: bank gathers are
bit-identical to record gathers, also under eviction).

* decode through a bank too small for the context (constant eviction) gives outputs and routing
  bit-identical to the bank-less RAM tier and to the VRAM tier;
* every resident bank slot holds exactly the record's rows of its group;
* the replacement policy is exact LRU (stamp, then slot index), checked step by step against a
  host model, and the hit / miss counters equal the model's.
"""
import pytest
import torch

import cases
from oracle import hga_oracle as O

pytestmark = pytest.mark.gpu

SPEC = dict(H=8, KVH=2, Dh=128, C=64, gs=16, Kc=4, Kg=8, kf=1, kl=2)


def _store(dev, B, tier, bank_chunks=0):
    from hierarchicalglobalattention_b200 import ChunkPlacementPolicy, ChunkRouter, RouterConfig, VramKVCacheStore
    from hierarchicalglobalattention_b200.store_ram import RamKVCacheStore
    s = SPEC
    cfg = RouterConfig(nhead=s["H"], kv_heads=s["KVH"], head_dim=s["Dh"], chunk_size=s["C"], group_size=s["gs"],
                       topk_chunks=s["Kc"], topk_groups=s["Kg"], theta=1e4)
    pol = ChunkPlacementPolicy(keep_first=s["kf"], keep_last=s["kl"], first_token_level=True)
    kw = dict(compute_device=dev, policy=pol, kv_heads=s["KVH"], head_dim=s["Dh"], chunk_size=s["C"],
              groups_per_chunk=s["C"] // s["gs"], batch_size=B, dtype=torch.bfloat16)
    store = VramKVCacheStore(**kw) if tier == "vram" else RamKVCacheStore(vram_cache_chunks=bank_chunks, **kw)
    return ChunkRouter(cfg, store)


def _run(router, g, S0, steps):
    C = SPEC["C"]
    router.seed(0, g["k_rope"][:, :, :S0], g["k_raw"][:, :, :S0], g["v"][:, :, :S0])
    outs, routes = [], []
    for i in range(steps):
        p = S0 + i
        sl = slice(p, p + 1)
        rk = router.decode_block(0, g["q"][:, :, sl], g["k_rope"][:, :, sl], g["k_raw"][:, :, sl], g["v"][:, :, sl], p)
        routes.append({k: t.clone() for k, t in rk.routing.items()})
        outs.append(rk.attend(g["q"][:, :, sl]))
    assert router.expected_position(0) == S0 + steps and (S0 + steps) // C > S0 // C  # chunks were closed
    return torch.cat(outs, 2), routes


def _inputs(dev, B, S, seed=8):
    p = O.OracleParams(nhead=SPEC["H"], kv_heads=SPEC["KVH"], head_dim=SPEC["Dh"], chunk_size=SPEC["C"],
                       group_size=SPEC["gs"], topk_chunks=SPEC["Kc"], topk_groups=SPEC["Kg"], keep_first=SPEC["kf"],
                       keep_last=SPEC["kl"], theta=1e4)
    c = {"name": "bank", "dtype": torch.bfloat16, "B": B, "S": S, "seed": seed, "params": p}
    return {k: t.to(dev) for k, t in cases.make_inputs(c).items() if k not in ("cos", "sin")}


def test_banked_decode_is_bit_identical_under_eviction(cuda):
    B, S0, steps = 2, 1500, 150                  # 23 closed chunks = 92 groups; the bank holds 32
    g = _inputs(cuda, B, S0 + steps)
    ref_out, ref_routes = _run(_store(cuda, B, "vram"), g, S0, steps)
    raw_out, _ = _run(_store(cuda, B, "ram"), g, S0, steps)
    router = _store(cuda, B, "ram", bank_chunks=8)   # 8 chunks x 4 groups = 32 slots = (H/KVH) * Kg
    out, routes = _run(router, g, S0, steps)
    torch.cuda.synchronize()
    assert torch.equal(raw_out, ref_out)
    assert torch.equal(out, ref_out)
    for a, b in zip(routes, ref_routes):
        for k in a:
            assert torch.equal(a[k], b[k]), k
    store = router.store
    assert store.cache_misses > 0 and store.cache_hits > 0
    assert store.summary_hits > 0 and store.summary_misses == 0
    # every resident slot holds its group's record rows
    bk = store._bank[0]
    st = store.layer_buffers(0)
    gs = SPEC["gs"]
    sg = bk["slot_gid"].cpu()
    rk, rv = st.token_k.cpu(), st.token_v.cpu()
    bank_k, bank_v = bk["k"].cpu(), bk["v"].cpu()
    checked = 0
    for b in range(B):
        for h in range(SPEC["KVH"]):
            for s, gid in enumerate(sg[b, h].tolist()):
                if gid < 0:
                    continue
                assert torch.equal(bank_k[b, h, s * gs:(s + 1) * gs], rk[b, h, gid * gs:(gid + 1) * gs])
                assert torch.equal(bank_v[b, h, s * gs:(s + 1) * gs], rv[b, h, gid * gs:(gid + 1) * gs])
                assert int(bk["gid_slot"][b, h, gid]) == s
                checked += 1
    assert checked == B * SPEC["KVH"] * bk["slots"]


def test_gather_h2d_is_exact_lru(cuda):
    """Random open lists over several steps against a host model of the bank: same slot maps, same
    hit / miss counts, bank rows equal to the record rows."""
    from hierarchicalglobalattention_b200 import _lib, ops
    B, H, KVH, Dh, gs, Kg = 2, 4, 2, 64, 16, 6
    rep = H // KVH
    n_slots, ngroups = 14, 40
    hp = _lib.make_params(batch=B, nhead=H, kv_heads=KVH, head_dim=Dh, chunk_size=64, group_size=gs, topk_chunks=4,
                          topk_groups=Kg, keep_first=0, keep_last=0, theta=1e4, dtype=torch.bfloat16)
    gen = torch.Generator().manual_seed(3)
    rec_k = torch.randn(B, KVH, ngroups * gs, Dh, generator=gen).to(torch.bfloat16).pin_memory()
    rec_v = torch.randn(B, KVH, ngroups * gs, Dh, generator=gen).to(torch.bfloat16).pin_memory()
    bank_k = torch.zeros(B, KVH, n_slots * gs, Dh, dtype=torch.bfloat16, device=cuda)
    bank_v = torch.zeros_like(bank_k)
    slot_gid = torch.full((B, KVH, n_slots), -1, dtype=torch.int32, device=cuda)
    slot_stamp = torch.full((B, KVH, n_slots), -1, dtype=torch.int32, device=cuda)
    gid_slot = torch.full((B, KVH, ngroups), -1, dtype=torch.int32, device=cuda)
    counters = torch.zeros(2, dtype=torch.int64, device=cuda)
    model = {(b, h): {"slot_gid": [-1] * n_slots, "stamp": [-1] * n_slots} for b in range(B) for h in range(KVH)}
    hits = misses = 0
    for step in range(12):
        # a hot set that drifts, so hits, misses and evictions all occur
        lo = (step * 3) % (ngroups - 12)
        og = torch.full((B, H, Kg), -1, dtype=torch.int32)
        for b in range(B):
            for h in range(H):
                pick = torch.randperm(12, generator=gen)[:Kg - (h % 2)] + lo
                og[b, h, :len(pick)] = pick.sort().values.to(torch.int32)
        open_slot = ops.gather_h2d(hp, og.to(cuda), rec_k, rec_v, bank_k, bank_v, slot_gid, gid_slot, slot_stamp, step,
                                   counters)
        torch.cuda.synchronize()
        for b in range(B):
            for kv in range(KVH):
                m = model[(b, kv)]
                uniq = sorted({int(x) for hh in range(kv * rep, (kv + 1) * rep) for x in og[b, hh].tolist() if x >= 0})
                g2s = {gg: s for s, gg in enumerate(m["slot_gid"]) if gg >= 0}
                miss = [gg for gg in uniq if gg not in g2s]
                for gg in uniq:
                    if gg in g2s:
                        m["stamp"][g2s[gg]] = step
                hits += len(uniq) - len(miss)
                misses += len(miss)
                # victims: the len(miss) smallest (stamp, slot); misses (ascending group) fill them
                # in the kernel's order: slots below the threshold stamp first, then those at it,
                # each run by slot index
                lru = sorted((st, s) for s, st in enumerate(m["stamp"]) if st != step)[:len(miss)]
                thr = lru[-1][0] if lru else 0
                order = sorted(lru, key=lambda x: (x[0] == thr, x[1]))
                for gg, (_, s) in zip(miss, order):
                    m["slot_gid"][s] = gg
                    m["stamp"][s] = step
                assert slot_gid[b, kv].tolist() == m["slot_gid"], (step, b, kv)
                assert slot_stamp[b, kv].tolist() == m["stamp"], (step, b, kv)
                for hh in range(kv * rep, (kv + 1) * rep):
                    for j, gg in enumerate(og[b, hh].tolist()):
                        want = m["slot_gid"].index(gg) if gg >= 0 else -1
                        assert int(open_slot[b, hh, j]) == want
        assert counters.tolist() == [hits, misses]
    bk, bv = bank_k.cpu(), bank_v.cpu()
    for b in range(B):
        for kv in range(KVH):
            for s, gg in enumerate(model[(b, kv)]["slot_gid"]):
                if gg >= 0:
                    assert torch.equal(bk[b, kv, s * gs:(s + 1) * gs], rec_k[b, kv, gg * gs:(gg + 1) * gs])
                    assert torch.equal(bv[b, kv, s * gs:(s + 1) * gs], rec_v[b, kv, gg * gs:(gg + 1) * gs])
