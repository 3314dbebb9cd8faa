"""Golden cases: seeded input generation shared by the fixture generator and the tests.

Inputs are regenerated from the seed with torch's CPU generator (deterministic for a given
torch build); every fixture stores a checksum of its inputs so RNG drift is detected.
"""
from __future__ import annotations

import math
import os
import sys

import torch

_ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
if _ROOT not in sys.path:
    sys.path.insert(0, _ROOT)
from oracle.hga_oracle import OracleParams, module_rotary  # noqa: E402

BF16, F32 = torch.bfloat16, torch.float32


def _p(**kw):
    return OracleParams(**kw)


CASES = [
    dict(name="sum_bf16", kind="summary", dtype=BF16, seed=11, B=1, S=1000,
         params=_p(nhead=4, kv_heads=4, head_dim=128, chunk_size=64, group_size=16, theta=1e6)),
    dict(name="sum_fp32", kind="summary", dtype=F32, seed=12, B=2, S=1000,
         params=_p(nhead=2, kv_heads=2, head_dim=64, chunk_size=64, group_size=16, theta=1e4)),
    dict(name="pf_tiny_fp32", kind="prefill", dtype=F32, seed=13, B=2, S=37,
         params=_p(nhead=4, kv_heads=2, head_dim=16, chunk_size=8, group_size=4, topk_chunks=2,
                   topk_groups=4, keep_first=1, keep_last=1, theta=1e4)),
    dict(name="pf_prev_fp32", kind="prefill", dtype=F32, seed=14, B=1, S=300,
         params=_p(nhead=4, kv_heads=2, head_dim=32, chunk_size=16, group_size=4, topk_chunks=3,
                   topk_groups=6, keep_first=0, keep_last=0, theta=1e4)),
    dict(name="pf_prev_bf16", kind="prefill", dtype=BF16, seed=15, B=1, S=300,
         params=_p(nhead=4, kv_heads=1, head_dim=64, chunk_size=16, group_size=4, topk_chunks=3,
                   topk_groups=6, keep_first=0, keep_last=0, theta=1e4)),
    dict(name="pf_cfg0", kind="prefill", dtype=F32, seed=16, B=1, S=4096, row_step=8,
         params=_p(nhead=8, kv_heads=2, head_dim=64, chunk_size=64, group_size=16, topk_chunks=16,
                   topk_groups=64, keep_first=2, keep_last=8, theta=1e4)),
    dict(name="pf_qwen_bf16", kind="prefill", dtype=BF16, seed=17, B=1, S=4096, row_step=16,
         params=_p(nhead=32, kv_heads=4, head_dim=128, chunk_size=64, group_size=16, topk_chunks=16,
                   topk_groups=64, keep_first=2, keep_last=8, theta=1e6)),
    dict(name="inc_tiny_fp32", kind="incremental", dtype=F32, seed=18, B=2, S=45, block=8,
         params=_p(nhead=4, kv_heads=2, head_dim=16, chunk_size=8, group_size=4, topk_chunks=2,
                   topk_groups=4, keep_first=1, keep_last=1, theta=1e4)),
    dict(name="inc_bf16", kind="incremental", dtype=BF16, seed=19, B=1, S=200, block=5,
         params=_p(nhead=8, kv_heads=2, head_dim=64, chunk_size=16, group_size=4, topk_chunks=3,
                   topk_groups=6, keep_first=1, keep_last=2, theta=1e4)),
    dict(name="mod_cfg0", kind="module", dtype=F32, seed=20, B=1, S=4096, row_step=8, d_model=512,
         params=_p(nhead=8, kv_heads=2, head_dim=64, chunk_size=64, group_size=16, topk_chunks=16,
                   topk_groups=64, keep_first=2, keep_last=8, theta=1e4)),
    # Qwen3 wrapper over HF Qwen3MoeAttention: a chunk-parallel prefill of `prefix` tokens, then
    # blocks of `block` tokens through the incremental path (the reference's serving schedule).
    # theta 1e6: the reference reads config.rope_theta, absent under transformers 5, and falls back
    # to 1e6, so the routed summaries agree only when the model's theta is 1e6 as well.
    dict(name="qwen_wrap_fp32", kind="qwen", dtype=F32, seed=21, B=1, S=1100, prefix=1024, block=19, row_step=3,
         d_model=512, params=_p(nhead=8, kv_heads=2, head_dim=64, chunk_size=64, group_size=16, topk_chunks=4,
                                topk_groups=8, keep_first=1, keep_last=2, theta=1e6)),
    # Dual Chunk Attention of the Qwen3 wrapper (dca_chunk > 0): pre-RoPE q / k and v fed as a
    # `prefix` call and then `block`-token calls (qwen_routed_attention.py:210-283).
    dict(name="dca_fp32", kind="dca", dtype=F32, seed=22, B=1, S=300, prefix=100, block=7, dca_chunk=32,
         dca_local=8, params=_p(nhead=4, kv_heads=2, head_dim=32, chunk_size=16, group_size=4, topk_chunks=3,
                                topk_groups=6, keep_first=1, keep_last=2, theta=1e4)),
    dict(name="dca_bf16", kind="dca", dtype=BF16, seed=23, B=2, S=400, prefix=130, block=5, dca_chunk=64, row_step=4,
         dca_local=12, params=_p(nhead=8, kv_heads=2, head_dim=64, chunk_size=16, group_size=4, topk_chunks=3,
                                 topk_groups=6, keep_first=1, keep_last=2, theta=1e4)),
]


def case(name):
    for c in CASES:
        if c["name"] == name:
            return c
    raise KeyError(name)


def rope_apply(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    half = x.shape[-1] // 2
    xf = x.float()
    return (xf * cos + torch.cat((-xf[..., half:], xf[..., :half]), dim=-1) * sin).to(x.dtype)


def make_inputs(c):
    """q/k_rope [B,H|KVH,S,Dh] RoPE'd in fp32 like the module; cos/sin = table in the model dtype."""
    p, B, S, dtype = c["params"], c["B"], c["S"], c["dtype"]
    g = torch.Generator().manual_seed(c["seed"])
    H, KVH, Dh = p.nhead, p.kv_heads, p.head_dim
    q_raw = torch.randn(B, H, S, Dh, generator=g).to(dtype)
    k_raw = torch.randn(B, KVH, S, Dh, generator=g).to(dtype)
    v = torch.randn(B, KVH, S, Dh, generator=g).to(dtype)
    cos, sin = module_rotary(p.theta, Dh, S)
    return {"q": rope_apply(q_raw, cos, sin), "k_rope": rope_apply(k_raw, cos, sin), "k_raw": k_raw,
            "v": v, "cos": cos.to(dtype), "sin": sin.to(dtype)}


def make_dca_inputs(c):
    """Pre-RoPE q [B,H,S,Dh], k_raw and v [B,KVH,S,Dh], N(0, 1) in the case dtype."""
    p, B, S, dtype = c["params"], c["B"], c["S"], c["dtype"]
    g = torch.Generator().manual_seed(c["seed"])
    H, KVH, Dh = p.nhead, p.kv_heads, p.head_dim
    return {"q": torch.randn(B, H, S, Dh, generator=g).to(dtype),
            "k_raw": torch.randn(B, KVH, S, Dh, generator=g).to(dtype),
            "v": torch.randn(B, KVH, S, Dh, generator=g).to(dtype)}


def make_module_inputs(c):
    """x and weights N(0, 0.02) (the config-0 recipe), norms absent unless qk_norm."""
    p, B, S, dtype, D = c["params"], c["B"], c["S"], c["dtype"], c["d_model"]
    g = torch.Generator().manual_seed(c["seed"])
    H, KVH, Dh = p.nhead, p.kv_heads, p.head_dim
    w = lambda o, i: (torch.randn(o, i, generator=g) * 0.02).to(dtype)  # noqa: E731
    return {"x": (torch.randn(B, S, D, generator=g) * 0.02).to(dtype),
            "wq": w(H * Dh, D), "wk": w(KVH * Dh, D), "wv": w(KVH * Dh, D), "wo": w(D, H * Dh)}


def make_qwen_inputs(c):
    """x N(0, 1), projections N(0, 0.02), q/k RMSNorm weights 1 + N(0, 0.1).  (Input checksums are
    fp32 sums whose order follows the host thread count: compare them at rel 1e-6.)"""
    p, B, S, dtype, D = c["params"], c["B"], c["S"], c["dtype"], c["d_model"]
    g = torch.Generator().manual_seed(c["seed"])
    H, KVH, Dh = p.nhead, p.kv_heads, p.head_dim
    w = lambda o, i: (torch.randn(o, i, generator=g) * 0.02).to(dtype)  # noqa: E731
    return {"x": torch.randn(B, S, D, generator=g).to(dtype),
            "wq": w(H * Dh, D), "wk": w(KVH * Dh, D), "wv": w(KVH * Dh, D), "wo": w(D, H * Dh),
            "qn": (1 + 0.1 * torch.randn(Dh, generator=g)).to(dtype),
            "kn": (1 + 0.1 * torch.randn(Dh, generator=g)).to(dtype)}


def qwen_config(c):
    """The HF Qwen3-MoE config of a qwen case (eager attention)."""
    from transformers import Qwen3MoeConfig
    p = c["params"]
    cfg = Qwen3MoeConfig(hidden_size=c["d_model"], num_attention_heads=p.nhead, num_key_value_heads=p.kv_heads,
                         head_dim=p.head_dim, num_hidden_layers=1, num_experts=4, num_experts_per_tok=2,
                         rms_norm_eps=1e-6, rope_theta=p.theta, attention_bias=False,
                         max_position_embeddings=max(4096, c["S"]))
    cfg._attn_implementation = "eager"
    return cfg


def load_qwen_weights(attn, inp):
    with torch.no_grad():
        attn.q_proj.weight.copy_(inp["wq"])
        attn.k_proj.weight.copy_(inp["wk"])
        attn.v_proj.weight.copy_(inp["wv"])
        attn.o_proj.weight.copy_(inp["wo"])
        attn.q_norm.weight.copy_(inp["qn"])
        attn.k_norm.weight.copy_(inp["kn"])


def qwen_schedule(c):
    """(lo, hi) blocks of a qwen case's forward calls."""
    blocks = [(0, c["prefix"])]
    s = c["prefix"]
    while s < c["S"]:
        blocks.append((s, min(s + c["block"], c["S"])))
        s = blocks[-1][1]
    return blocks


def load_module_weights(m, inp):
    with torch.no_grad():
        m.q_proj.weight.copy_(inp["wq"])
        m.k_proj.weight.copy_(inp["wk"])
        m.v_proj.weight.copy_(inp["wv"])
        m.o_proj.weight.copy_(inp["wo"])


def output_rows(c, S):
    step = c.get("row_step", 1)
    rows = list(range(0, S, step))
    if rows[-1] != S - 1:
        rows.append(S - 1)
    return torch.tensor(rows, dtype=torch.long)


def checksum(inp) -> float:
    tot = 0.0
    for k in sorted(inp):
        t = inp[k].float()
        tot += float(t.abs().sum()) * (1 + len(k)) + float((t * torch.arange(t.numel()).view_as(t).remainder(7)).sum())
    return tot


def fixture_path(name):
    return os.path.join(os.path.dirname(os.path.abspath(__file__)), f"{name}.pt")


def load(name):
    return torch.load(fixture_path(name), weights_only=False)


__all__ = ["CASES", "case", "make_inputs", "make_dca_inputs", "make_module_inputs", "make_qwen_inputs", "qwen_config",
           "load_qwen_weights", "qwen_schedule", "output_rows", "checksum", "load",
           "rope_apply", "math"]
