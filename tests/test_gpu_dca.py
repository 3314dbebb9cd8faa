"""GPU parity of the Dual Chunk Attention path (the Qwen3 wrapper's dca_chunk > 0 variant,
qwen_routed_attention.py:210-283): intra-chunk-roped keys routed through the incremental decode
router and attended by the DCA decode kernel (hga_attend_decode_dca), against the reference's
golden outputs, the CPU oracle and through the Qwen3 wrapper module."""
import types

import pytest
import torch

import cases
from oracle import hga_oracle as O

pytestmark = pytest.mark.gpu

TIERS = ["vram", "ram", "ram_nobank"]


def _router(p, B, dtype, dev, tier):
    from hierarchicalglobalattention_b200 import ChunkPlacementPolicy, ChunkRouter, RouterConfig, VramKVCacheStore
    from hierarchicalglobalattention_b200.store_ram import RamKVCacheStore
    cfg = RouterConfig(nhead=p.nhead, kv_heads=p.kv_heads, head_dim=p.head_dim, chunk_size=p.chunk_size,
                       group_size=p.group_size, topk_chunks=p.topk_chunks, topk_groups=p.topk_groups, theta=p.theta)
    policy = ChunkPlacementPolicy(keep_first=p.keep_first, keep_last=p.keep_last, first_token_level=True)
    kw = dict(compute_device=dev, policy=policy, kv_heads=p.kv_heads, head_dim=p.head_dim, chunk_size=p.chunk_size,
              groups_per_chunk=p.chunk_size // p.group_size, batch_size=B, dtype=dtype)
    if tier == "vram":
        store = VramKVCacheStore(**kw)
    else:
        store = RamKVCacheStore(vram_cache_chunks=0 if tier == "ram_nobank" else 256, **kw)
    return ChunkRouter(cfg, store)


def _keep(blocks, shape):
    """(b, h, row) not decided by a near tie of the routing (located by the oracle)."""
    keep = torch.ones(shape, dtype=torch.bool)
    for blk in blocks:
        keep[:, :, blk["pos"]:blk["pos"] + blk["L"]] &= ~blk["route"]["tie"].unsqueeze(-1)
    return keep


@pytest.mark.parametrize("tier", TIERS)
@pytest.mark.parametrize("name", [c["name"] for c in cases.CASES if c["kind"] == "dca"])
def test_dca_matches_reference_golden(cuda, name, tier):
    from hierarchicalglobalattention_b200.qwen import dca_forward
    c, gold = cases.case(name), cases.load(name)
    p = c["params"]
    inp = cases.make_dca_inputs(c)
    assert cases.checksum(inp) == pytest.approx(gold["input_checksum"], rel=1e-6)
    sched = cases.qwen_schedule(c)
    _, blocks = O.dca_sequence(p, inp["q"], inp["k_raw"], inp["v"], c["dca_chunk"], c["dca_local"], sched)
    g = {k: t.to(cuda) for k, t in inp.items()}
    router = _router(p, c["B"], c["dtype"], cuda, tier)
    ceil = c["dca_chunk"] + c["dca_local"]
    outs = []
    with torch.no_grad():
        for lo, hi in sched:
            outs.append(dca_forward(router, 0, g["q"][:, :, lo:hi], g["k_raw"][:, :, lo:hi], g["v"][:, :, lo:hi], lo,
                                    c["dca_chunk"], ceil, p.theta))
    out = torch.cat(outs, dim=2).cpu()
    rows = gold["out_rows"]
    k = _keep(blocks, out.shape[:3])[:, :, rows]
    assert k.float().mean() > 0.8
    tol = 1e-4 if c["dtype"] == torch.float32 else 2e-2
    torch.testing.assert_close(out[:, :, rows][k].float(), gold["out"][k].float(), atol=tol, rtol=tol)


@pytest.mark.parametrize("dca_chunk,dca_local,block", [(128, 24, 1), (64, 0, 9), (256, 40, 64)])
def test_dca_decode_vs_oracle_bf16_qwen_shape(cuda, dca_chunk, dca_local, block):
    """Qwen3-like head shape (Dh 128, GQA 4:1, C 64, group 16) in bf16 over ~1.3K tokens: a prefix
    call and then blocks, against the oracle restatement on every untied (block, head)."""
    p = O.OracleParams(nhead=8, kv_heads=2, head_dim=128, chunk_size=64, group_size=16, topk_chunks=4,
                       topk_groups=8, keep_first=1, keep_last=2, theta=1e6)
    B, S, prefix = 2, 1300, 700
    local = dca_local if dca_local > 0 else max(1, dca_chunk // 5)
    c = {"params": p, "B": B, "S": S, "seed": 31, "dtype": torch.bfloat16}
    inp = cases.make_dca_inputs(c)
    sched = [(0, prefix)] + [(s, min(s + block, S)) for s in range(prefix, S, block)]
    ref, blocks = O.dca_sequence(p, inp["q"], inp["k_raw"], inp["v"], dca_chunk, local, sched, tie_rule="index")
    from hierarchicalglobalattention_b200.qwen import dca_forward
    g = {k: t.to(cuda) for k, t in inp.items()}
    router = _router(p, B, torch.bfloat16, cuda, "vram")
    with torch.no_grad():
        out = torch.cat([dca_forward(router, 0, g["q"][:, :, lo:hi], g["k_raw"][:, :, lo:hi], g["v"][:, :, lo:hi], lo,
                                     dca_chunk, dca_chunk + local, p.theta) for lo, hi in sched], dim=2).cpu()
    k = _keep(blocks, out.shape[:3])
    assert k.float().mean() > 0.8
    torch.testing.assert_close(out[k].float(), ref[k].float(), atol=2e-2, rtol=2e-2)


def test_dca_route_query_block_segments(cuda):
    """route_query_block(..., return_positions=True) gives the incremental segments the DCA caller
    attends in order (VRAM tier), identical to the chunk-by-chunk helper."""
    from hierarchicalglobalattention_b200.qwen import dca_forward, dca_rotate
    from hierarchicalglobalattention_b200 import ops
    c = cases.case("dca_fp32")
    p = c["params"]
    inp = {k: t.to(cuda) for k, t in cases.make_dca_inputs(c).items()}
    S, L_c, ceil = 100, c["dca_chunk"], c["dca_chunk"] + c["dca_local"]
    q, k_raw, v = inp["q"][:, :, :S], inp["k_raw"][:, :, :S], inp["v"][:, :, :S]
    r1 = _router(p, c["B"], c["dtype"], cuda, "vram")
    want = dca_forward(r1, 0, q, k_raw, v, 0, L_c, ceil, p.theta)
    r2 = _router(p, c["B"], c["dtype"], cuda, "vram")
    pos = torch.arange(S, device=cuda)
    tc, ts = ops.dca_rope_table(ceil, p.head_dim, p.theta, cuda)
    cs, sn = tc[pos % L_c], ts[pos % L_c]
    segs = r2.route_query_block(0, dca_rotate(q, cs, sn), dca_rotate(k_raw, cs, sn), k_raw, v, 0,
                                return_positions=True)
    assert [(lo, hi) for _, lo, hi in segs] == [(i, min(i + p.chunk_size, S)) for i in range(0, S, p.chunk_size)]
    got = torch.cat([rk.attend_dca(q[:, :, lo:hi], pos[lo:hi], L_c, ceil, p.theta) for rk, lo, hi in segs], dim=2)
    assert torch.equal(got, want)


def test_qwen_wrapper_dca_vs_oracle(cuda):
    """QwenRoutedAttention(dca_chunk > 0) over HF Qwen3MoeAttention weights (fused prologue kernel
    with the intra-chunk RoPE rows, DCA attention kernel, o_proj) against the oracle's DCA on the
    HF layers' own q/k norms and projections, fed as a prefix call and then 5-token calls."""
    from transformers import Qwen3MoeConfig
    from transformers.models.qwen3_moe.modeling_qwen3_moe import Qwen3MoeAttention, Qwen3MoeRotaryEmbedding
    from hierarchicalglobalattention_b200.qwen import QwenRoutedAttention
    torch.manual_seed(0)
    cfg = Qwen3MoeConfig(hidden_size=256, num_attention_heads=4, num_key_value_heads=2, head_dim=64,
                         num_hidden_layers=1, num_experts=4, num_experts_per_tok=2, rms_norm_eps=1e-6,
                         rope_theta=1e6, attention_bias=False, max_position_embeddings=4096)
    attn = Qwen3MoeAttention(cfg, layer_idx=0).to(device=cuda, dtype=torch.float32).eval()
    with torch.no_grad():
        attn.q_norm.weight.normal_(1.0, 0.1)
        attn.k_norm.weight.normal_(1.0, 0.1)
    rot = Qwen3MoeRotaryEmbedding(cfg).to(cuda)
    S, prefix, blk, C, L_c = 400, 150, 5, 16, 64
    x = torch.randn(1, S, cfg.hidden_size, device=cuda)
    pos = torch.arange(S, device=cuda).unsqueeze(0)
    cos, sin = rot(x, pos)
    w = QwenRoutedAttention(attn, cfg, keep_first=1, keep_last=2, topk_chunks=3, topk_groups=6, chunk_size=C,
                            group_size=4, dca_chunk=L_c)
    assert w.dca_local == L_c // 5 and w.dca_ceil == L_c + L_c // 5
    pkv = types.SimpleNamespace()
    sched = [(0, prefix)] + [(s, min(s + blk, S)) for s in range(prefix, S, blk)]
    with torch.no_grad():
        got = torch.cat([w(x[:, lo:hi], position_embeddings=(cos[:, lo:hi], sin[:, lo:hi]), attention_mask=None,
                           past_key_values=pkv, position_ids=pos[:, lo:hi])[0] for lo, hi in sched], dim=1)
        H, KVH, Dh = 4, 2, 64
        q = attn.q_norm(attn.q_proj(x).view(1, S, H, Dh)).transpose(1, 2).cpu()
        k = attn.k_norm(attn.k_proj(x).view(1, S, KVH, Dh)).transpose(1, 2).cpu()
        v = attn.v_proj(x).view(1, S, KVH, Dh).transpose(1, 2).cpu()
        p = O.OracleParams(nhead=H, kv_heads=KVH, head_dim=Dh, chunk_size=C, group_size=4, topk_chunks=3,
                           topk_groups=6, keep_first=1, keep_last=2, theta=1e6)
        heads, blocks = O.dca_sequence(p, q, k, v, L_c, L_c // 5, sched, tie_rule="index")
        keep = _keep(blocks, heads.shape[:3])
        assert keep.all(), "fp32 case expected free of routing ties"
        want = attn.o_proj(heads.transpose(1, 2).reshape(1, S, H * Dh).to(cuda))
    torch.testing.assert_close(got, want, atol=2e-4, rtol=2e-4)
