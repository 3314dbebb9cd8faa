"""The Qwen3 patch (QwenRoutedAttention over HF Qwen3MoeAttention) on the B200 kernels: against
the reference wrapper's own outputs (sparse routing, prefill + incremental blocks) and, at full
coverage, against the stock HF attention (the reference's selftest_wrapper_vs_qwen bar)."""
import types

import pytest
import torch

import cases

pytestmark = pytest.mark.gpu


def _hf(c, dev, dtype):
    from transformers.models.qwen3_moe.modeling_qwen3_moe import Qwen3MoeAttention, Qwen3MoeRotaryEmbedding
    cfg = cases.qwen_config(c)
    attn = Qwen3MoeAttention(cfg, layer_idx=0).to(device=dev, dtype=dtype).eval()
    return cfg, attn, Qwen3MoeRotaryEmbedding(cfg).to(dev)


@pytest.mark.parametrize("tier", ["vram", "ram"])
def test_wrapper_matches_reference_golden(cuda, tier):
    from hierarchicalglobalattention_b200.qwen import QwenRoutedAttention
    c, gold = cases.case("qwen_wrap_fp32"), cases.load("qwen_wrap_fp32")
    p = c["params"]
    inp = cases.make_qwen_inputs(c)
    assert cases.checksum(inp) == pytest.approx(gold["input_checksum"], rel=1e-6)
    cfg, attn, rot = _hf(c, cuda, c["dtype"])
    cases.load_qwen_weights(attn, {k: t.to(cuda) for k, t in inp.items()})
    x = inp["x"].to(cuda)
    S = x.shape[1]
    pos = torch.arange(S, device=cuda).unsqueeze(0)
    cos, sin = rot(x, pos)
    w = QwenRoutedAttention(attn, cfg, keep_first=p.keep_first, keep_last=p.keep_last, topk_chunks=p.topk_chunks,
                            topk_groups=p.topk_groups, chunk_size=p.chunk_size, group_size=p.group_size,
                            cache_location=tier)
    pkv = types.SimpleNamespace()
    outs = []
    with torch.no_grad():
        for lo, hi in cases.qwen_schedule(c):
            o, none = w(x[:, lo:hi], position_embeddings=(cos[:, lo:hi], sin[:, lo:hi]), attention_mask=None,
                        past_key_values=pkv, position_ids=pos[:, lo:hi])
            assert none is None
            outs.append(o)
    out = torch.cat(outs, dim=1)[:, gold["out_rows"]].cpu()
    torch.testing.assert_close(out, gold["out"], atol=1e-4, rtol=1e-4)
    assert hasattr(pkv, "_kv_router")


@pytest.mark.parametrize("realistic", [False, True], ids=["tiny-fp32", "realistic-bf16"])
def test_wrapper_full_coverage_equals_hf_attention(cuda, realistic):
    """keep_last covering every chunk: the routed wrapper is exact attention (single call and
    blocked calls sharing a cache-attached router)."""
    from transformers import Qwen3MoeConfig
    from transformers.models.qwen3_moe.modeling_qwen3_moe import Qwen3MoeAttention, Qwen3MoeRotaryEmbedding
    from hierarchicalglobalattention_b200.qwen import QwenRoutedAttention
    torch.manual_seed(0)
    if realistic:
        cfg = Qwen3MoeConfig(hidden_size=2048, num_attention_heads=32, num_key_value_heads=4, head_dim=128,
                             num_hidden_layers=1, num_experts=4, num_experts_per_tok=2, rms_norm_eps=1e-6,
                             rope_theta=10_000_000.0, attention_bias=False, max_position_embeddings=262144)
        S, C, gs, dtype, tol = 200, 64, 16, torch.bfloat16, 0.05
    else:
        cfg = Qwen3MoeConfig(hidden_size=128, num_attention_heads=8, num_key_value_heads=2, head_dim=16,
                             num_hidden_layers=1, num_experts=4, num_experts_per_tok=2, rms_norm_eps=1e-6,
                             rope_theta=10000.0, attention_bias=False, max_position_embeddings=4096)
        S, C, gs, dtype, tol = 20, 8, 4, torch.float32, 1e-3
    cfg._attn_implementation = "sdpa"
    attn = Qwen3MoeAttention(cfg, layer_idx=0).to(device=cuda, dtype=dtype).eval()
    with torch.no_grad():
        attn.q_norm.weight.normal_(1.0, 0.1)
        attn.k_norm.weight.normal_(1.0, 0.1)
    rot = Qwen3MoeRotaryEmbedding(cfg).to(cuda)
    x = torch.randn(1, S, cfg.hidden_size, device=cuda, dtype=dtype)
    pos = torch.arange(S, device=cuda).unsqueeze(0)
    cos, sin = rot(x, pos)
    causal = torch.triu(torch.full((S, S), float("-inf"), device=cuda, dtype=dtype), diagonal=1).view(1, 1, S, S)
    with torch.no_grad():
        ref, _ = attn(x, position_embeddings=(cos, sin), attention_mask=causal, past_key_values=None)
        w = QwenRoutedAttention(attn, cfg, keep_first=0, keep_last=9999, topk_chunks=0, chunk_size=C, group_size=gs)
        out, _ = w(x, position_embeddings=(cos, sin), attention_mask=None, position_ids=pos)
        w2 = QwenRoutedAttention(attn, cfg, keep_first=0, keep_last=9999, topk_chunks=0, chunk_size=C, group_size=gs)
        pkv = types.SimpleNamespace()
        outs = []
        for s in range(0, S, 16):
            e = min(s + 16, S)
            ob, _ = w2(x[:, s:e], position_embeddings=(cos[:, s:e], sin[:, s:e]), attention_mask=None,
                       past_key_values=pkv, position_ids=pos[:, s:e])
            outs.append(ob)
        out_blk = torch.cat(outs, dim=1)
    assert (out - ref).abs().max().item() < tol
    assert (out_blk - ref).abs().max().item() < tol


def test_patch_a_model_and_restore(cuda):
    """replace_qwen_attention_with_router on a 2-layer Qwen3-MoE model: generation-style calls run
    through the routed layers; restore puts the original modules back."""
    from transformers import Qwen3MoeConfig, Qwen3MoeForCausalLM
    from transformers.cache_utils import DynamicCache
    from hierarchicalglobalattention_b200.qwen import (QwenRoutedAttention, replace_qwen_attention_with_router,
                                                       restore_original_attention)
    torch.manual_seed(0)
    cfg = Qwen3MoeConfig(vocab_size=512, hidden_size=256, intermediate_size=256, moe_intermediate_size=128,
                         num_attention_heads=4, num_key_value_heads=2, head_dim=64, num_hidden_layers=2,
                         num_experts=4, num_experts_per_tok=2, rope_theta=1e6, max_position_embeddings=4096)
    model = Qwen3MoeForCausalLM(cfg).to(device=cuda, dtype=torch.bfloat16).eval()
    origs = [layer.self_attn for layer in model.model.layers]
    n_params = sum(p.numel() for p in model.parameters())
    assert replace_qwen_attention_with_router(model, keep_first=1, keep_last=2, topk_chunks=4, topk_groups=8) == 2
    assert all(isinstance(layer.self_attn, QwenRoutedAttention) for layer in model.model.layers)
    assert sum(p.numel() for p in model.parameters()) == n_params
    ids = torch.randint(0, 512, (1, 300), device=cuda)
    with torch.no_grad():
        cache = DynamicCache(config=cfg)
        out = model(input_ids=ids, past_key_values=cache, use_cache=True)
        nxt = out.logits[:, -1:].argmax(-1)
        out2 = model(input_ids=nxt, past_key_values=cache, use_cache=True)
    assert torch.isfinite(out.logits.float()).all() and torch.isfinite(out2.logits.float()).all()
    assert restore_original_attention(model) == 2
    assert [layer.self_attn for layer in model.model.layers] == origs
