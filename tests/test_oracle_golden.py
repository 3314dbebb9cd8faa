"""The CPU oracle reproduces the reference's own outputs (tests/golden, made by make_golden.py)."""
import pytest
import torch

import cases
from oracle import hga_oracle as O


def _sets_from_gold(g, C, M, B, H, N):
    d = {}
    for b in range(B):
        for h in range(H):
            for n in range(N):
                c, gg = {}, {}
                if "chunk_idx" in g:
                    for j in range(g["chunk_idx"].shape[-1]):
                        t0 = int(g["chunk_t0"][b, h, n, j])
                        if t0 < C:
                            c[int(g["chunk_idx"][b, h, n, j])] = t0
                if "group_chunk" in g:
                    for j in range(g["group_chunk"].shape[-1]):
                        t0 = int(g["group_t0"][b, h, n, j])
                        if t0 < C:
                            gg[int(g["group_chunk"][b, h, n, j]) * M + int(g["group_idx"][b, h, n, j])] = t0
                d[(b, h, n)] = (c, gg)
    return d


@pytest.mark.parametrize("name", [c["name"] for c in cases.CASES if c["kind"] == "summary"])
def test_summaries_match_reference(name):
    c, g = cases.case(name), cases.load(name)
    inp = cases.make_inputs(c)
    assert cases.checksum(inp) == pytest.approx(g["input_checksum"], rel=1e-6)
    ck, gk, _ = O.summaries_prefill(c["params"], inp["k_raw"], inp["k_rope"], inp["v"], inp["cos"], inp["sin"])
    assert torch.equal(ck, g["chunk_k"]) and torch.equal(gk, g["group_k"])


@pytest.mark.parametrize("name", [c["name"] for c in cases.CASES if c["kind"] == "prefill"
                                  and c["S"] <= 1024])
def test_prefill_routing_and_output_match_reference(name):
    c, g = cases.case(name), cases.load(name)
    p, S = c["params"], c["S"]
    inp = cases.make_inputs(c)
    assert cases.checksum(inp) == pytest.approx(g["input_checksum"], rel=1e-6)
    ck, gk, _ = O.summaries_prefill(p, inp["k_raw"], inp["k_rope"], inp["v"], inp["cos"], inp["sin"])
    r = O.route_prefill(p, inp["q"], ck, gk, S)
    B, H = inp["q"].shape[:2]
    N = (S + p.chunk_size - 1) // p.chunk_size
    assert O.visible_sets(r, p.chunk_size, p.M) == _sets_from_gold(g, p.chunk_size, p.M, B, H, N)
    out = O.attend_prefill(p, inp["q"], inp["k_rope"], inp["v"], r, S)
    tol = 1e-5 if c["dtype"] == torch.float32 else 2e-2
    assert (out[:, :, g["out_rows"]].float() - g["out"].float()).abs().max().item() < tol


def test_module_forward_matches_reference_cfg0_rows():
    """Config-0 module forward (fp32) on a sample of query chunks vs the reference module."""
    c, g = cases.case("mod_cfg0"), cases.load("mod_cfg0")
    p = c["params"]
    inp = cases.make_module_inputs(c)
    S = c["S"]
    chunks = [0, 1, 9, 10, 33, 63]
    out, _ = O.module_forward(p, inp["x"], inp["wq"], inp["wk"], inp["wv"], inp["wo"], None, None, 1e-6,
                              chunks=chunks)
    rows = g["out_rows"]
    keep = torch.tensor([int(r) // p.chunk_size in chunks for r in rows])
    err = (out[:, rows[keep]] - g["out"][:, keep]).abs().max().item()
    assert err < 1e-6


@pytest.mark.parametrize("name", [c["name"] for c in cases.CASES if c["kind"] == "incremental"])
def test_incremental_decode_matches_reference(name):
    """Block-by-block decode (chunk_router.py:279-442) with its closed-chunk summaries."""
    c, g = cases.case(name), cases.load(name)
    inp = cases.make_inputs(c)
    assert cases.checksum(inp) == pytest.approx(g["input_checksum"], rel=1e-6)
    out, blocks = O.decode_sequence(c["params"], inp["q"], inp["k_rope"], inp["k_raw"], inp["v"], c["block"])
    n = g["store_chunk_k"].shape[2]
    ck, _, _ = O.summaries_store(c["params"], inp["k_raw"], inp["k_rope"], inp["v"])
    assert torch.equal(ck[:, :, :n], g["store_chunk_k"])
    tol = 1e-5 if c["dtype"] == torch.float32 else 2e-2
    torch.testing.assert_close(out[:, :, g["out_rows"]].float(), g["out"].float(), atol=tol, rtol=tol)


@pytest.mark.parametrize("name", [c["name"] for c in cases.CASES if c["kind"] == "dca"])
def test_dca_matches_reference(name):
    """Dual Chunk Attention of the Qwen3 wrapper (qwen_routed_attention.py:210-283): intra-chunk
    keys routed through the incremental path, three query ropings chosen per key."""
    c, g = cases.case(name), cases.load(name)
    inp = cases.make_dca_inputs(c)
    assert cases.checksum(inp) == pytest.approx(g["input_checksum"], rel=1e-6)
    out, _ = O.dca_sequence(c["params"], inp["q"], inp["k_raw"], inp["v"], c["dca_chunk"], c["dca_local"],
                            cases.qwen_schedule(c))
    tol = 1e-5 if c["dtype"] == torch.float32 else 2e-2
    torch.testing.assert_close(out[:, :, g["out_rows"]].float(), g["out"].float(), atol=tol, rtol=tol)
