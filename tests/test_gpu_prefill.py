"""GPU parity of the prefill hot path (summary builder, router, working-set attention) against the
CPU oracle and the reference's golden outputs.  All calls go through the C ABI (libhga_b200.so)."""
import pytest
import torch
import torch.nn.functional as F

import cases
import hga_check as HC
from oracle import hga_oracle as O

pytestmark = pytest.mark.gpu

PREFILL_CASES = [c["name"] for c in cases.CASES if c["kind"] == "prefill"]


def _params(c, dtype=None):
    from hierarchicalglobalattention_b200 import _lib
    p = c["params"]
    return _lib.make_params(batch=c["B"], nhead=p.nhead, kv_heads=p.kv_heads, head_dim=p.head_dim,
                            chunk_size=p.chunk_size, group_size=p.group_size, topk_chunks=p.topk_chunks,
                            topk_groups=p.topk_groups, keep_first=p.keep_first, keep_last=p.keep_last,
                            theta=p.theta, dtype=dtype or c["dtype"])


def _gpu_pipeline(c, inp, dev, impl=0, debug=True):
    from hierarchicalglobalattention_b200 import ops
    hp = _params(c)
    g = {k: v.to(dev) for k, v in inp.items()}
    ck, gk, gv = ops.summaries(hp, g["k_raw"], g["k_rope"], g["v"], g["cos"], g["sin"])
    res = ops.route_prefill(hp, g["q"], ck, gk, debug=debug)
    out = ops.attend_prefill(hp, g["q"], g["k_rope"], g["v"], res["open_gid"], res["open_t0"], impl=impl)
    torch.cuda.synchronize()
    return ck, gk, gv, res, out


@pytest.mark.parametrize("name", ["sum_bf16", "sum_fp32"])
def test_summaries_bit_exact_vs_reference(cuda, name):
    from hierarchicalglobalattention_b200 import ops
    c, g = cases.case(name), cases.load(name)
    inp = {k: v.to(cuda) for k, v in cases.make_inputs(c).items()}
    ck, gk, gv = ops.summaries(_params(c), inp["k_raw"], inp["k_rope"], inp["v"], inp["cos"], inp["sin"])
    assert torch.equal(ck.cpu(), g["chunk_k"])
    assert torch.equal(gk.cpu(), g["group_k"])
    # group V sums vs the oracle restatement
    _, _, ogv = O.summaries_prefill(c["params"], *(cases.make_inputs(c)[k] for k in ("k_raw", "k_rope", "v", "cos", "sin")))
    assert torch.equal(gv.cpu(), ogv)


@pytest.mark.parametrize("name", PREFILL_CASES)
def test_router_selection_replays_exactly(cuda, name):
    """Given the kernel's own rounded scores, its selections are exactly the reference rules."""
    c = cases.case(name)
    inp = cases.make_inputs(c)
    ck, gk, _, res, _ = _gpu_pipeline(c, inp, cuda)
    bad, _ = HC.check_replay(c["params"], c["S"], res)
    assert not bad, f"{len(bad)} tiles differ from the replay, e.g. {bad[:3]}"


@pytest.mark.parametrize("name", PREFILL_CASES)
def test_router_scores_within_reference_rounding(cuda, name):
    c = cases.case(name)
    inp = cases.make_inputs(c)
    ck, gk, _, res, _ = _gpu_pipeline(c, inp, cuda)
    assert HC.check_scores_in_bounds(c["params"], c["S"], inp["q"], ck, gk, res) == 0


@pytest.mark.parametrize("name", PREFILL_CASES)
def test_router_and_output_vs_reference(cuda, name):
    """Visible chunk/group sets equal the reference's except on flagged near-tie tiles; the output
    rows of the reference golden file match within the dtype tolerance on the agreeing tiles."""
    c, gold = cases.case(name), cases.load(name)
    p, S = c["params"], c["S"]
    inp = cases.make_inputs(c)
    _, _, _, res, out = _gpu_pipeline(c, inp, cuda)
    ck, gk, _ = O.summaries_prefill(p, inp["k_raw"], inp["k_rope"], inp["v"], inp["cos"], inp["sin"])
    oroute = O.route_prefill(p, inp["q"], ck, gk, S)
    osets = HC.oracle_sets(oroute, p.chunk_size, p.M)
    gsets = HC.gpu_sets(res, p.M)
    mism = [k for k in osets if osets[k] != gsets[k]]
    unexplained = [k for k in mism if not bool(oroute["tie"][k])]
    assert not unexplained, f"{len(unexplained)} non-tie tiles differ, e.g. {unexplained[:3]}"
    print(f"\n[{name}] tiles {len(osets)}, differing (all flagged) {len(mism)}, "
          f"flagged {int(oroute['tie'].sum())}")
    # fp32: flagged ties are rare; bf16: the reference's own torch.topk order among equal bf16
    # scores decides many tiles (implementation-defined; measured 9% differing at pf_qwen_bf16)
    assert len(mism) <= (max(1, len(osets) // 50) if c["dtype"] == torch.float32 else len(osets) * 0.2)
    # outputs on agreeing tiles vs the reference's golden rows
    rows = gold["out_rows"]
    C = p.chunk_size
    bad_tiles = {(b, h, n) for (b, h, n) in mism}
    B, H = inp["q"].shape[:2]
    tol_abs, tol_rel = HC.TOL[c["dtype"]]
    o = out.cpu()[:, :, rows]
    ref = gold["out"]
    keep = torch.ones_like(ref, dtype=torch.bool)
    for (b, h, n) in bad_tiles:
        sel = (rows // C) == n
        keep[b, h, sel] = False
    d = (o.float() - ref.float()).abs()[keep]
    assert d.max().item() < tol_abs
    assert (d.sum() / ref.float().abs()[keep].sum()).item() < tol_rel


@pytest.mark.parametrize("name", PREFILL_CASES)
def test_router_sets_vs_index_rule_oracle(cuda, name):
    """Strict set parity: the oracle run under the kernels' tie rule (equal scores: lower index)
    agrees on every tile except those an accumulation-order difference could flip, and those are
    capped (fp32 5%, bf16 35%)."""
    c = cases.case(name)
    p, S = c["params"], c["S"]
    inp = cases.make_inputs(c)
    _, _, _, res, _ = _gpu_pipeline(c, inp, cuda)
    ck, gk, _ = O.summaries_prefill(p, inp["k_raw"], inp["k_rope"], inp["v"], inp["cos"], inp["sin"])
    r = O.route_prefill(p, inp["q"], ck, gk, S, tie_rule="index")
    rep = HC.tie_report(HC.oracle_sets(r, p.chunk_size, p.M), HC.gpu_sets(res, p.M), r["tie"])
    print(f"\n[{name}] index-rule parity: tiles {rep['tiles']}, differing {rep['mismatch']}, "
          f"flagged {rep['tie_frac']:.3f}")
    assert not rep["unexplained"], f"non-tie tiles differ, e.g. {rep['unexplained'][:3]}"
    assert rep["tie_frac"] <= (0.05 if c["dtype"] == torch.float32 else 0.35)


@pytest.mark.parametrize("name", PREFILL_CASES)
@pytest.mark.parametrize("impl", [0, 1])
def test_attention_vs_oracle_on_gpu_routing(cuda, name, impl):
    c = cases.case(name)
    p, S = c["params"], c["S"]
    inp = cases.make_inputs(c)
    _, _, _, res, out = _gpu_pipeline(c, inp, cuda, impl=impl)
    route = HC.route_dict_from_gpu(res, p, S)
    ref = O.attend_prefill(p, inp["q"], inp["k_rope"], inp["v"], route, S)
    mx, rel = HC.attn_errors(out.cpu(), ref, c["dtype"])
    tol_abs, tol_rel = HC.TOL[c["dtype"]]
    assert mx < tol_abs and rel < tol_rel, (mx, rel)


@pytest.mark.parametrize("S", [1, 7, 8, 9, 37, 64])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_full_window_equals_dense_causal(cuda, S, dtype):
    """keep_last covering everything and no routing == dense causal attention (the reference's
    selftest_exact_equivalence, test_qwen30b_routed.py:80-143), including S=1 and ragged tails."""
    p = O.OracleParams(nhead=4, kv_heads=2, head_dim=16, chunk_size=8, group_size=4, topk_chunks=0,
                       topk_groups=0, keep_first=0, keep_last=10_000, theta=1e4)
    c = dict(name="dense", kind="prefill", dtype=dtype, seed=3, B=1, S=S, params=p)
    inp = cases.make_inputs(c)
    _, _, _, res, out = _gpu_pipeline(c, inp, cuda, impl=1, debug=False)
    q = inp["q"].float()
    k = inp["k_rope"].float().repeat_interleave(2, dim=1)
    v = inp["v"].float().repeat_interleave(2, dim=1)
    ref = F.scaled_dot_product_attention(q, k, v, is_causal=True)
    tol = 1e-5 if dtype == torch.float32 else 2e-2
    assert (out.cpu().float() - ref).abs().max().item() < tol


def test_router_empty_pool_and_ragged_tail(cuda):
    """First chunks (empty routed pool) and a 1-token last chunk produce empty / valid lists."""
    p = O.OracleParams(nhead=2, kv_heads=1, head_dim=32, chunk_size=16, group_size=4, topk_chunks=2,
                       topk_groups=4, keep_first=1, keep_last=1, theta=1e4)
    c = dict(name="ragged", kind="prefill", dtype=torch.float32, seed=5, B=2, S=16 * 6 + 1, params=p)
    inp = cases.make_inputs(c)
    _, _, _, res, out = _gpu_pipeline(c, inp, cuda)
    sel = res["sel_chunk"].cpu()
    assert (sel[:, :, :3] == -1).all()          # chunks 0..2: pool empty (keep_first=1, keep_last=1)
    assert (sel[:, :, 3:] >= 0).any()
    bad, _ = HC.check_replay(p, c["S"], res)
    assert not bad
    assert torch.isfinite(out.cpu()).all()


@pytest.mark.parametrize("dtype,dh,S", [(torch.bfloat16, 128, 1000), (torch.bfloat16, 64, 257), (torch.float16, 128, 640)])
def test_summaries_dual_equals_two_single_calls(cuda, dtype, dh, S):
    """hga_summaries_dual (one read of K/V) writes the routing set and the store seed bit-identical
    to the two hga_summaries calls it replaces, ragged last chunk included."""
    from hierarchicalglobalattention_b200 import _lib, ops
    g = torch.Generator().manual_seed(dh + S)
    B, KVH, C, gs = 2, 2, 64, 16
    k_raw, k_rope, v = (torch.randn(B, KVH, S, dh, generator=g).to(dtype).to(cuda) for _ in range(3))
    hp = _lib.make_params(batch=B, nhead=4, kv_heads=KVH, head_dim=dh, chunk_size=C, group_size=gs, topk_chunks=4,
                          topk_groups=8, keep_first=1, keep_last=2, theta=1e4, dtype=dtype)
    cos_a, sin_a = (t.to(cuda) for t in O.module_rotary(1e4, dh, S))
    cos_b, sin_b = (t.to(cuda) * (1 + 1e-3) for t in O.module_rotary(1e4, dh, S))   # a different table
    n_b = S // C
    cap = n_b + 3
    ref_b = [torch.zeros(B, KVH, cap, dh, dtype=dtype, device=cuda), torch.zeros(B, KVH, cap, 4, dh, dtype=dtype, device=cuda),
             torch.zeros(B, KVH, cap, 4, dh, dtype=dtype, device=cuda)]
    got_b = [t.clone() for t in ref_b]
    ck_a, gk_a, _ = ops.summaries(hp, k_raw, k_rope, v, cos_a, sin_a, round_table=True, with_group_v=False)
    ops.summaries(hp, k_raw, k_rope, v, cos_b, sin_b, seq_len=n_b * C, out=tuple(ref_b), out_chunk0=0)
    ck_d, gk_d = ops.summaries_dual(hp, k_raw, k_rope, v, cos_a, sin_a, cos_b, sin_b, tuple(got_b), n_b, round_a=True)
    torch.cuda.synchronize()
    assert torch.equal(ck_d, ck_a) and torch.equal(gk_d, gk_a)
    for a, b in zip(got_b, ref_b):
        assert torch.equal(a, b)


def test_torch_ops_match_the_c_abi_calls(cuda):
    """torch.ops.hga.* run the same kernels as the ops wrappers (bit-identical results)."""
    from hierarchicalglobalattention_b200 import ops, torch_ops
    c = cases.case("pf_qwen_bf16")
    inp = {k: v.to(cuda) for k, v in cases.make_inputs(c).items()}
    hp = _params(c)
    pi, pf = torch_ops.params_lists(hp)
    ck, gk, _ = ops.summaries(hp, inp["k_raw"], inp["k_rope"], inp["v"], inp["cos"], inp["sin"])
    ck2, gk2, _ = torch.ops.hga.summaries(pi, pf, inp["k_raw"], inp["k_rope"], inp["v"], inp["cos"], inp["sin"], False)
    assert torch.equal(ck, ck2) and torch.equal(gk, gk2)
    r = ops.route_prefill(hp, inp["q"], ck, gk)
    sc, st, og, ot = torch.ops.hga.route_prefill(pi, pf, inp["q"], ck, gk)
    assert torch.equal(sc, r["sel_chunk"]) and torch.equal(og, r["open_gid"]) and torch.equal(ot, r["open_t0"])
    out = ops.attend_prefill(hp, inp["q"], inp["k_rope"], inp["v"], og, ot)
    out2 = torch.ops.hga.attend_prefill(pi, pf, inp["q"], inp["k_rope"], inp["v"], og, ot)
    assert torch.equal(out.transpose(1, 2), out2)
