"""tcgen05 router (impl 2): selection replay from its own scores, score bounds, agreement with the
portable router and with the reference selections (near ties excepted)."""
import pytest
import torch

import cases
import hga_check as HC
from oracle import hga_oracle as O

pytestmark = pytest.mark.gpu

CASES = [
    # (S, B, H, KVH, kf, kl, topk_chunks, topk_groups, q_layout)
    (4096, 1, 32, 4, 2, 8, 16, 64, 1),     # configs[1] routing at 4K
    (1000, 2, 8, 2, 0, 0, 3, 6, 0),        # prev forcing, ragged tail, Kg < Kc*M (pooled group choice)
    (8192, 1, 8, 2, 2, 8, 32, 128, 1),     # configs[3] routing parameters (Kc 32, Kg_request 64)
    (300, 1, 2, 1, 1, 1, 20, 32, 1),       # Kc > pool for early chunks
    (2048, 1, 8, 2, 1, 4, 16, 100, 1),     # top-16 lists with 50 requests of 64: one thread per row, radix select
    (1500, 1, 4, 1, 1, 2, 4, 64, 1),       # requests cover every candidate (Kg_request >= Kc * M)
]


def _route(case, impl, cuda, debug=True):
    from hierarchicalglobalattention_b200 import _lib, ops
    S, B, H, KVH, kf, kl, kc, kg, ql = case
    p = O.OracleParams(nhead=H, kv_heads=KVH, head_dim=128, chunk_size=64, group_size=16, topk_chunks=kc,
                       topk_groups=kg, keep_first=kf, keep_last=kl, theta=1e6)
    c = dict(dtype=torch.bfloat16, seed=S + H, B=B, S=S, params=p)
    inp = cases.make_inputs(c)
    g = {k: v.to(cuda) for k, v in inp.items()}
    hp = _lib.make_params(batch=B, nhead=H, kv_heads=KVH, head_dim=128, chunk_size=64, group_size=16,
                          topk_chunks=kc, topk_groups=kg, keep_first=kf, keep_last=kl, theta=1e6,
                          dtype=torch.bfloat16)
    ck, gk, _ = ops.summaries(hp, g["k_raw"], g["k_rope"], g["v"], g["cos"], g["sin"])
    q = g["q"] if ql == 0 else g["q"].transpose(1, 2).contiguous().transpose(1, 2)
    res = ops.route_prefill(hp, q, ck, gk, debug=debug, impl=impl)
    torch.cuda.synchronize()
    assert _lib.device_status() == 0
    return p, inp, ck.cpu(), gk.cpu(), res


@pytest.mark.parametrize("case", CASES)
def test_tc_router_replay_and_bounds(cuda, case):
    p, inp, ck, gk, res = _route(case, 2, cuda)
    bad, _ = HC.check_replay(p, case[0], res)
    assert not bad, f"{len(bad)} tiles differ from the replay, e.g. {bad[:3]}"
    assert HC.check_scores_in_bounds(p, case[0], inp["q"], ck, gk, res) == 0


@pytest.mark.parametrize("case", CASES)
def test_tc_router_vs_reference(cuda, case):
    p, inp, ck, gk, res = _route(case, 2, cuda, debug=False)
    S = case[0]
    oroute = O.route_prefill(p, inp["q"], ck, gk, S)
    osets = HC.oracle_sets(oroute, 64, 4)
    gsets = HC.gpu_sets(res, 4)
    mism = [k for k in osets if osets[k] != gsets[k]]
    unexplained = [k for k in mism if not bool(oroute["tie"][k])]
    assert not unexplained, f"{len(unexplained)} non-tie tiles differ, e.g. {unexplained[:3]}"


def test_tc_router_matches_portable_router_on_its_scores(cuda):
    """Both kernels, fed the same inputs, agree wherever their dumped scores agree."""
    case = CASES[0]
    _, _, _, _, r2 = _route(case, 2, cuda)
    _, _, _, _, r1 = _route(case, 1, cuda)
    same = torch.isclose(r1["dbg_l1"], r2["dbg_l1"], equal_nan=True).all(dim=-1).all(dim=-1)
    same &= torch.isclose(r1["dbg_l2"], r2["dbg_l2"], equal_nan=True).all(dim=-1).all(dim=-1)
    eq = (r1["sel_chunk"] == r2["sel_chunk"]).all(-1) & (r1["sel_t0"] == r2["sel_t0"]).all(-1)
    eq &= (r1["open_gid"] == r2["open_gid"]).all(-1) & (r1["open_t0"] == r2["open_t0"]).all(-1)
    assert bool(eq[same].all())
    assert same.float().mean().item() > 0.5


@pytest.mark.parametrize("S,H,KVH,kf,kl,tc_,tg", [(700, 4, 1, 1, 1, 3, 4), (600, 2, 1, 0, 0, 3, 6), (200, 2, 1, 0, 1, 3, 12)])
def test_tc_router_is_deterministic_when_groups_outnumber_chunks(cuda, S, H, KVH, kf, kl, tc_, tg):
    """Level 2 reuses the level-1 per-chunk arrays for topk_chunks * M group keys, which can exceed
    the number of chunks on short sequences; repeated calls must give identical lists."""
    from hierarchicalglobalattention_b200 import _lib, ops
    p = O.OracleParams(nhead=H, kv_heads=KVH, head_dim=128, chunk_size=64, group_size=16, topk_chunks=tc_,
                       topk_groups=tg, keep_first=kf, keep_last=kl, theta=1e6)
    c = dict(dtype=torch.bfloat16, seed=5, B=1, S=S, params=p)
    inp = {k: v.to(cuda) for k, v in cases.make_inputs(c).items()}
    hp = _lib.make_params(batch=1, nhead=H, kv_heads=KVH, head_dim=128, chunk_size=64, group_size=16,
                          topk_chunks=tc_, topk_groups=tg, keep_first=kf, keep_last=kl, theta=1e6,
                          dtype=torch.bfloat16)
    ck, gk, _ = ops.summaries(hp, inp["k_raw"], inp["k_rope"], inp["v"], inp["cos"], inp["sin"])
    runs = [ops.route_prefill(hp, inp["q"], ck, gk, impl=2) for _ in range(6)]
    for r in runs:
        for k in r:
            assert torch.equal(r[k], runs[0][k]), k
