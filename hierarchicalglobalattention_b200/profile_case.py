"""Run the prefill kernels once on a seeded Qwen3-30B-shaped case (for ncu captures).

    python -m hierarchicalglobalattention_b200.profile_case --seq 8192

Builds random RoPE'd q / k and v (bf16, 32 query heads, 4 KV heads, head_dim 128), then runs
hga_summaries, hga_route_prefill and hga_attend_prefill (tensor-core kernels) ``--reps`` times.
``--decode B`` instead seeds a VRAM store with B sequences of ``--seq`` tokens and runs one-token
hga_route_decode + hga_attend_decode steps (the configs[2] decode shape).
"""
from __future__ import annotations

import argparse

import torch

from . import _lib, ops


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--seq", type=int, default=8192)
    ap.add_argument("--reps", type=int, default=2)
    ap.add_argument("--topk-chunks", type=int, default=16)
    ap.add_argument("--topk-groups", type=int, default=64)
    ap.add_argument("--decode", type=int, default=0, help="batch of a decode case (0: prefill case)")
    args = ap.parse_args()
    if args.decode:
        return decode_case(args)
    dev = torch.device("cuda:0")
    S, H, KVH, Dh = args.seq, 32, 4, 128
    g = torch.Generator(device="cpu").manual_seed(1)
    half = Dh // 2
    inv = 1.0 / (1e6 ** (torch.arange(half, dtype=torch.float32) / half))
    f = torch.arange(S, dtype=torch.float32)[:, None] * inv
    cos, sin = torch.cat((f, f), -1).cos(), torch.cat((f, f), -1).sin()

    def rope(x):
        xf = x.float()
        return (xf * cos + torch.cat((-xf[..., half:], xf[..., :half]), -1) * sin).to(torch.bfloat16)

    q = rope(torch.randn(1, H, S, Dh, generator=g).to(torch.bfloat16))
    k_raw = torch.randn(1, KVH, S, Dh, generator=g).to(torch.bfloat16)
    v = torch.randn(1, KVH, S, Dh, generator=g).to(torch.bfloat16)
    k_rope = rope(k_raw)
    q = q.transpose(1, 2).contiguous().to(dev).transpose(1, 2)
    k_raw, k_rope, v, cos, sin = (t.to(dev) for t in (k_raw, k_rope, v, cos, sin))
    hp = _lib.make_params(batch=1, nhead=H, kv_heads=KVH, head_dim=Dh, chunk_size=64, group_size=16,
                          topk_chunks=args.topk_chunks, topk_groups=args.topk_groups, keep_first=2,
                          keep_last=8, theta=1e6, dtype=torch.bfloat16)
    ck, gk, _ = ops.summaries(hp, k_raw, k_rope, v, cos, sin, round_table=True)
    for _ in range(args.reps):
        res = ops.route_prefill(hp, q, ck, gk, impl=2)
        ops.attend_prefill(hp, q, k_rope, v, res["open_gid"], res["open_t0"], impl=2)
    torch.cuda.synchronize()
    print("ok, device status", _lib.device_status())


def decode_case(args) -> None:
    from .config import ChunkPlacementPolicy, RouterConfig
    from .router import ChunkRouter
    from .store import VramKVCacheStore
    dev = torch.device("cuda:0")
    B, S, H, KVH, Dh = args.decode, args.seq, 32, 4, 128
    g = torch.Generator(device=dev).manual_seed(0)
    cfg = RouterConfig(nhead=H, kv_heads=KVH, head_dim=Dh, chunk_size=64, group_size=16,
                       topk_chunks=args.topk_chunks, topk_groups=args.topk_groups, theta=1e6)
    pol = ChunkPlacementPolicy(keep_first=2, keep_last=8, first_token_level=True)
    store = VramKVCacheStore(compute_device=dev, policy=pol, kv_heads=KVH, head_dim=Dh, chunk_size=64,
                             groups_per_chunk=4, batch_size=B, dtype=torch.bfloat16)
    router = ChunkRouter(cfg, store)
    k = torch.randn(B, KVH, S, Dh, device=dev, dtype=torch.bfloat16, generator=g)
    router.seed(0, k, k, k)
    store.ensure_capacity(0, S // 64 + 1, S + 64)
    hp = cfg.hga_params(pol, B, torch.bfloat16)
    st = store.layer_buffers(0)
    q = torch.randn(B, H, 1, Dh, device=dev, dtype=torch.bfloat16, generator=g)
    seq = torch.full((B,), S, dtype=torch.int32, device=dev)
    for _ in range(args.reps):
        r = ops.route_decode(hp, q, seq, st.chunk_k, st.group_k, S // 64 - 10)
        ops.attend_decode(hp, q, seq, st.token_k, st.token_v, 0, st.token_k, st.token_v, r["open_gid"], r["open_t0"])
    torch.cuda.synchronize()
    print("ok, device status", _lib.device_status())


if __name__ == "__main__":
    main()
