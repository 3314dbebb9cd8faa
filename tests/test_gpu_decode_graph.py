"""A decode step replayed from a CUDA graph (DecodeStepGraph) equals ChunkRouter.decode_step run
eagerly on the same mixed-length batch, across chunk closes, on both store tiers and two layers."""
import pytest
import torch

import cases
from oracle import hga_oracle as O

pytestmark = pytest.mark.gpu

SHAPES = [
    # (dtype, H, KVH, Dh, Kc, Kg, kf, kl, tolerance)
    (torch.bfloat16, 8, 2, 128, 4, 8, 1, 2, 2e-2),
    (torch.float32, 4, 2, 64, 8, 16, 1, 4, 1e-4),
]


def _router(p, B, dtype, dev, tier):
    from hierarchicalglobalattention_b200 import ChunkPlacementPolicy, ChunkRouter, RouterConfig, VramKVCacheStore
    from hierarchicalglobalattention_b200.store_ram import RamKVCacheStore
    cfg = RouterConfig(nhead=p.nhead, kv_heads=p.kv_heads, head_dim=p.head_dim, chunk_size=p.chunk_size,
                       group_size=p.group_size, topk_chunks=p.topk_chunks, topk_groups=p.topk_groups, theta=p.theta)
    policy = ChunkPlacementPolicy(keep_first=p.keep_first, keep_last=p.keep_last, first_token_level=True)
    cls = VramKVCacheStore if tier == "vram" else RamKVCacheStore
    store = cls(compute_device=dev, policy=policy, kv_heads=p.kv_heads, head_dim=p.head_dim,
                chunk_size=p.chunk_size, groups_per_chunk=p.chunk_size // p.group_size, batch_size=B, dtype=dtype)
    return ChunkRouter(cfg, store)


@pytest.mark.parametrize("tier", ["vram", "ram"])
@pytest.mark.parametrize("shape", SHAPES, ids=["bf16", "fp32"])
def test_graph_decode_equals_eager_decode_step(cuda, tier, shape):
    from hierarchicalglobalattention_b200.decode_graph import DecodeStepGraph
    dtype, H, KVH, Dh, Kc, Kg, kf, kl, tol = shape
    p = O.OracleParams(nhead=H, kv_heads=KVH, head_dim=Dh, chunk_size=64, group_size=16, topk_chunks=Kc,
                       topk_groups=Kg, keep_first=kf, keep_last=kl, theta=1e4)
    starts = [130, 700, 1023, 1290]     # a short pool, mid-chunk, about to close, further on
    steps, layers = 70, 2
    B, Smax = len(starts), max(starts)
    inp = cases.make_inputs({"dtype": dtype, "B": layers, "S": Smax + steps, "seed": 11, "params": p})
    g = {k: t.to(cuda) for k, t in inp.items()}          # batch row = layer; every sequence shares it

    def fresh():
        r = _router(p, B, dtype, cuda, tier)
        for layer in range(layers):
            r.seed_mixed(layer, *(g[k][layer:layer + 1, :, :Smax].expand(B, -1, -1, -1).contiguous()
                                  for k in ("k_rope", "k_raw", "v")), starts)
        return r

    def token(layer, pos_host, name):
        idx = torch.tensor(pos_host, device=cuda)
        return g[name][layer][:, idx].permute(1, 0, 2).unsqueeze(2).contiguous()    # [B,heads,1,Dh]

    eager, pos = fresh(), list(starts)
    ref = []
    for _ in range(steps):
        seq = torch.tensor(pos, dtype=torch.int32, device=cuda)
        per = []
        for layer in range(layers):
            qb = token(layer, pos, "q")
            rk = eager.decode_step(layer, qb, token(layer, pos, "k_rope"), token(layer, pos, "k_raw"),
                                   token(layer, pos, "v"), seq, pos)
            per.append(rk.attend(qb, use_summaries=False))
        ref.append(torch.stack(per))
        pos = [x + 1 for x in pos]

    router = fresh()
    graph = DecodeStepGraph(router, range(layers), list(starts), capacity_tokens=Smax + steps + 1, dtype=dtype)
    pos = list(starts)
    for i in range(steps):
        for layer in range(layers):
            graph.q[layer].copy_(token(layer, pos, "q"))
            graph.k_rope[layer].copy_(token(layer, pos, "k_rope"))
            graph.k_raw[layer].copy_(token(layer, pos, "k_raw"))
            graph.v[layer].copy_(token(layer, pos, "v"))
        out = graph.step()
        torch.testing.assert_close(out.float(), ref[i].float(), atol=tol, rtol=tol,
                                   msg=lambda m: f"step {i}: {m}")
        pos = [x + 1 for x in pos]
    assert graph.seq_pos.tolist() == pos


def test_graph_refuses_positions_past_capacity(cuda):
    from hierarchicalglobalattention_b200.decode_graph import DecodeStepGraph
    p = O.OracleParams(nhead=4, kv_heads=2, head_dim=64, chunk_size=64, group_size=16, topk_chunks=4,
                       topk_groups=8, keep_first=1, keep_last=2, theta=1e4)
    router = _router(p, 1, torch.float32, cuda, "vram")
    with pytest.raises(ValueError):
        DecodeStepGraph(router, [0], [500], capacity_tokens=400, dtype=torch.float32)
