"""Module-level parity: HierarchicalGlobalAttentionRouted on the B200 kernels vs the reference."""
import pytest
import torch

import cases
from oracle import hga_oracle as O

pytestmark = pytest.mark.gpu


def _module(c, dtype, qk_norm=False):
    import hierarchicalglobalattention_b200 as hga
    p = c["params"]
    m = hga.HierarchicalGlobalAttentionRouted(d_model=c["d_model"], nhead=p.nhead, kv_heads=p.kv_heads,
                                              head_dim=p.head_dim, chunk_size=p.chunk_size,
                                              group_size=p.group_size, topk_chunks=p.topk_chunks,
                                              topk_groups=p.topk_groups, keep_first=p.keep_first,
                                              keep_last=p.keep_last, theta=p.theta, qk_norm=qk_norm)
    return m


def test_module_cfg0_matches_reference_golden(cuda):
    """configs[0] (fp32, S=4096) forward vs the reference module's output rows."""
    c, g = cases.case("mod_cfg0"), cases.load("mod_cfg0")
    inp = cases.make_module_inputs(c)
    m = _module(c, torch.float32)
    cases.load_module_weights(m, inp)
    m = m.to(cuda)
    with torch.no_grad():
        out, extra = m(inp["x"].to(cuda))
    assert extra == {}
    got = out.cpu()[:, g["out_rows"]]
    err = (got - g["out"]).abs().max().item()
    assert err < 1e-4 * max(1.0, g["out"].abs().max().item()), err


def _qwen_module(cuda, seed, **kw):
    import hierarchicalglobalattention_b200 as hga
    cfg = dict(d_model=2048, nhead=32, kv_heads=4, head_dim=128, chunk_size=64, group_size=16, topk_chunks=16,
               topk_groups=64, keep_first=2, keep_last=8, theta=1e6, qk_norm=True)
    cfg.update(kw)
    m = hga.HierarchicalGlobalAttentionRouted(**cfg)
    g = torch.Generator().manual_seed(seed)
    with torch.no_grad():
        for n, prm in m.named_parameters():
            if "norm" in n:
                prm.copy_(1.0 + 0.1 * torch.randn(prm.shape, generator=g))
            else:
                prm.copy_(torch.randn(prm.shape, generator=g) * 0.02)
    return m.to(torch.bfloat16), g


def _dense_reference(m, x):
    """Dense causal attention through the same projections / norms / RoPE (torch ops on the GPU)."""
    import torch.nn.functional as F
    B, S, _ = x.shape
    H, KVH, Dh = m.nhead, m.kv_heads, m.head_dim
    q = m.q_norm(m.q_proj(x).view(B, S, H, Dh)).transpose(1, 2)
    k = m.k_norm(m.k_proj(x).view(B, S, KVH, Dh)).transpose(1, 2)
    v = m.v_proj(x).view(B, S, KVH, Dh).transpose(1, 2)
    cos, sin = O.module_rotary(m.theta, Dh, S)
    cos, sin = cos.to(x.device), sin.to(x.device)
    qr = O._rotate(q.float(), cos, sin).to(x.dtype)
    kr = O._rotate(k.float(), cos, sin).to(x.dtype)
    rep = H // KVH
    o = F.scaled_dot_product_attention(qr.float(), kr.float().repeat_interleave(rep, 1),
                                       v.float().repeat_interleave(rep, 1), is_causal=True).to(x.dtype)
    return m.o_proj(o.transpose(1, 2).reshape(B, S, H * Dh))


@pytest.mark.parametrize("S,kl", [(1024, 16), (1000, 10_000), (200, 4)])
def test_module_qwen_shape_bf16_full_coverage_equals_dense(cuda, S, kl):
    """Everything kept token-level (keep_last covers the context, no routing) == dense causal
    attention: the reference's realistic wrapper self-test (test_qwen30b_routed.py:146-215, tol 0.05)."""
    m, g = _qwen_module(cuda, S, keep_first=0, keep_last=kl, topk_chunks=0, topk_groups=0)
    m = m.to(cuda)
    x = torch.randn(1, S, 2048, generator=g).to(torch.bfloat16).to(cuda)
    with torch.no_grad():
        out, _ = m(x)
        ref = _dense_reference(m, x)
    assert (out.float() - ref.float()).abs().max().item() < 0.05


@pytest.mark.parametrize("S", [1000, 2048])
def test_module_qwen_shape_bf16_sparse_vs_oracle(cuda, S):
    """Sparse routing at the Qwen3-30B layer shape vs the oracle's module forward on the same weights.
    CPU and GPU projections round differently, which moves near-tie routing decisions of a few
    (head, chunk) tiles; the bulk of the rows must agree within the bf16 tolerance."""
    p = O.OracleParams(nhead=32, kv_heads=4, head_dim=128, chunk_size=64, group_size=16, topk_chunks=16,
                       topk_groups=64, keep_first=2, keep_last=8, theta=1e6)
    m, g = _qwen_module(cuda, S)
    x = torch.randn(1, S, 2048, generator=g).to(torch.bfloat16)
    ref, _ = O.module_forward(p, x, m.q_proj.weight, m.k_proj.weight, m.v_proj.weight, m.o_proj.weight,
                              m.q_norm.weight, m.k_norm.weight, 1e-6)
    m = m.to(cuda)
    with torch.no_grad():
        out, _ = m(x.to(cuda))
    d = (out.cpu().float() - ref.float()).abs()
    row_err = d.amax(dim=-1).flatten()
    frac_bad = (row_err > 0.05).float().mean().item()
    mean_rel = (d.sum() / ref.float().abs().sum()).item()
    assert frac_bad < 0.05 and mean_rel < 2e-2, (frac_bad, mean_rel, row_err.max().item())


@pytest.mark.parametrize("tier", ["vram", "ram"])
def test_store_reuse_across_sequences(cuda, tier):
    """A store reset keeps its buffers (no re-allocation or zero fill): a longer sequence, then a
    shorter one, then a prefill followed by decode blocks, give the outputs of fresh modules."""
    import hierarchicalglobalattention_b200 as hga
    torch.manual_seed(3)
    kw = dict(d_model=512, nhead=8, kv_heads=2, head_dim=64, chunk_size=64, group_size=16, topk_chunks=4,
              topk_groups=8, keep_first=1, keep_last=2, theta=1e4, cache_location=tier)
    m = hga.HierarchicalGlobalAttentionRouted(**kw).to(cuda).to(torch.bfloat16)
    xs = [torch.randn(1, S, 512, device=cuda, dtype=torch.bfloat16) for S in (1500, 700)]

    def fresh(x):
        f = hga.HierarchicalGlobalAttentionRouted(**kw).to(cuda).to(torch.bfloat16)
        f.load_state_dict(m.state_dict())
        return f(x)[0]

    with torch.no_grad():
        for x in xs:
            assert torch.equal(m(x)[0], fresh(x))
        # prefill 640 tokens, then 3-token blocks on the reused store, against a fresh module
        x = torch.randn(1, 700, 512, device=cuda, dtype=torch.bfloat16)
        f = hga.HierarchicalGlobalAttentionRouted(**kw).to(cuda).to(torch.bfloat16)
        f.load_state_dict(m.state_dict())
        outs = []
        for mod in (m, f):
            o = [mod(x[:, :640], cache_position=torch.arange(640, device=cuda))[0]]
            for s in range(640, 700, 3):
                o.append(mod(x[:, s:s + 3], cache_position=torch.arange(s, s + 3, device=cuda))[0])
            outs.append(torch.cat(o, dim=1))
        assert torch.equal(outs[0], outs[1])
