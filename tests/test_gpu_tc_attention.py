"""tcgen05/TMEM attention kernel (impl 2) vs the portable SIMT kernel (impl 1) and the oracle."""
import pytest
import torch

import cases
import hga_check as HC
from oracle import hga_oracle as O

pytestmark = pytest.mark.gpu


def _run(S, B, H, KVH, kf, kl, topk_c, topk_g, q_layout, out_layout, seed, cuda):
    from hierarchicalglobalattention_b200 import _lib, ops
    p = O.OracleParams(nhead=H, kv_heads=KVH, head_dim=128, chunk_size=64, group_size=16, topk_chunks=topk_c,
                       topk_groups=topk_g, keep_first=kf, keep_last=kl, theta=1e6)
    c = dict(dtype=torch.bfloat16, seed=seed, B=B, S=S, params=p)
    inp = {k: v.to(cuda) for k, v in cases.make_inputs(c).items()}
    hp = _lib.make_params(batch=B, nhead=H, kv_heads=KVH, head_dim=128, chunk_size=64, group_size=16,
                          topk_chunks=topk_c, topk_groups=topk_g, keep_first=kf, keep_last=kl, theta=1e6,
                          dtype=torch.bfloat16)
    ck, gk, _ = ops.summaries(hp, inp["k_raw"], inp["k_rope"], inp["v"], inp["cos"], inp["sin"])
    q = inp["q"] if q_layout == 0 else inp["q"].transpose(1, 2).contiguous().transpose(1, 2)
    res = ops.route_prefill(hp, q, ck, gk)
    outs = {}
    for impl in (1, 2):
        outs[impl] = ops.attend_prefill(hp, q, inp["k_rope"], inp["v"], res["open_gid"], res["open_t0"],
                                        out_layout=out_layout, impl=impl)
    torch.cuda.synchronize()
    assert _lib.device_status() == 0
    return p, c, inp, res, outs


@pytest.mark.parametrize("S,B", [(64, 1), (130, 1), (1000, 2), (4096, 1)])
def test_tc_matches_simt(cuda, S, B):
    p, c, inp, res, outs = _run(S, B, 8, 2, 2, 8, 16, 64, 1, 1, 31 + S, cuda)
    mx, rel = HC.attn_errors(outs[2], outs[1], torch.bfloat16)
    assert mx < 2e-2 and rel < 5e-3, (mx, rel)


@pytest.mark.parametrize("q_layout,out_layout", [(0, 0), (0, 1), (1, 0)])
def test_tc_layouts(cuda, q_layout, out_layout):
    p, c, inp, res, outs = _run(700, 1, 4, 1, 1, 3, 4, 8, q_layout, out_layout, 5, cuda)
    mx, rel = HC.attn_errors(outs[2], outs[1], torch.bfloat16)
    assert mx < 2e-2 and rel < 5e-3, (mx, rel)


def test_tc_vs_oracle_qwen_routing(cuda):
    """Full Qwen3-30B head layout (32/4 heads) at S=2048 vs the oracle attention on the same routing."""
    p, c, inp, res, outs = _run(2048, 1, 32, 4, 2, 8, 16, 64, 1, 1, 77, cuda)
    route = HC.route_dict_from_gpu(res, p, 2048)
    cpu = {k: v.cpu() for k, v in inp.items()}
    ref = O.attend_prefill(p, cpu["q"], cpu["k_rope"], cpu["v"], route, 2048)
    mx, rel = HC.attn_errors(outs[2].cpu(), ref, torch.bfloat16)
    assert mx < 2e-2 and rel < 5e-3, (mx, rel)


def test_tc_no_routing_windows_only(cuda):
    """topk 0 (windows + causal only) and keep_first/keep_last 0 (causal chunk only)."""
    for kf, kl, tc_, tg in ((2, 8, 0, 0), (0, 0, 0, 0), (0, 0, 3, 6)):
        p, c, inp, res, outs = _run(600, 1, 2, 1, kf, kl, tc_, tg, 1, 1, 9, cuda)
        mx, rel = HC.attn_errors(outs[2], outs[1], torch.bfloat16)
        assert mx < 2e-2 and rel < 5e-3, (kf, kl, mx, rel)


def test_bounded_wait_runs_out_without_a_fault(cuda):
    """The failure path of the bounded waits: one CTA's K load is withheld (hga_debug_fault), its
    wait runs out after 1 ms, it records the code, drains and releases its TMEM; every other CTA
    finishes, and the next launch is clean and equal to a normal one."""
    from hierarchicalglobalattention_b200 import _lib, ops
    c = cases.case("pf_qwen_bf16")
    inp = {k: v.to(cuda) for k, v in cases.make_inputs(c).items()}
    p = c["params"]
    hp = _lib.make_params(batch=c["B"], nhead=p.nhead, kv_heads=p.kv_heads, head_dim=p.head_dim,
                          chunk_size=p.chunk_size, group_size=p.group_size, topk_chunks=p.topk_chunks,
                          topk_groups=p.topk_groups, keep_first=p.keep_first, keep_last=p.keep_last, theta=p.theta,
                          dtype=c["dtype"])
    ck, gk, _ = ops.summaries(hp, inp["k_raw"], inp["k_rope"], inp["v"], inp["cos"], inp["sin"])
    r = ops.route_prefill(hp, inp["q"], ck, gk)
    torch.cuda.synchronize()
    _lib.device_status(clear=True)
    ref = ops.attend_prefill(hp, inp["q"], inp["k_rope"], inp["v"], r["open_gid"], r["open_t0"], impl=2)
    torch.cuda.synchronize()
    assert _lib.device_status(clear=True) == 0
    assert _lib.lib().hga_debug_fault(1, 1_000_000) == 0
    bad = ops.attend_prefill(hp, inp["q"], inp["k_rope"], inp["v"], r["open_gid"], r["open_t0"], impl=2)
    torch.cuda.synchronize()
    # one of the stalled CTA's waits ran out first (codes 1-10 name the wait; which one wins the
    # race between its warps varies), never a drain (0x7f)
    code = _lib.device_status(clear=True)
    assert 1 <= code <= 10, code
    keep = torch.ones(bad.shape[:3], dtype=torch.bool, device=cuda)
    S, C = bad.shape[2], p.chunk_size
    keep[0, 0:2, (S - 1) // C * C:] = False                # CTA (last chunk, heads 0-1, batch 0) wrote nothing
    assert torch.equal(bad[keep], ref[keep])
    again = ops.attend_prefill(hp, inp["q"], inp["k_rope"], inp["v"], r["open_gid"], r["open_t0"], impl=2)
    torch.cuda.synchronize()
    assert _lib.device_status(clear=True) == 0
    assert torch.equal(again, ref)
