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


@pytest.mark.parametrize("S", [1000, 2048])
def test_module_qwen_shape_bf16_vs_oracle(cuda, S):
    """Qwen3-30B-shaped layer (qk_norm, bf16) vs the oracle's module forward on the same weights."""
    p = O.OracleParams(nhead=32, kv_heads=4, head_dim=128, chunk_size=64, group_size=16, topk_chunks=16,
                       topk_groups=64, keep_first=2, keep_last=8, theta=1e6)
    c = dict(params=p, d_model=2048)
    m = _module(c, torch.bfloat16, qk_norm=True)
    g = torch.Generator().manual_seed(S)
    with torch.no_grad():
        for n, prm in m.named_parameters():
            if "norm" in n:
                prm.copy_(1.0 + 0.1 * torch.randn(prm.shape, generator=g))
            else:
                prm.copy_(torch.randn(prm.shape, generator=g) * 0.02)
    m = m.to(torch.bfloat16)
    x = torch.randn(1, S, 2048, generator=g).to(torch.bfloat16)
    ref, _ = O.module_forward(p, x, m.q_proj.weight, m.k_proj.weight, m.v_proj.weight, m.o_proj.weight,
                              m.q_norm.weight, m.k_norm.weight, 1e-6)
    m = m.to(cuda)
    with torch.no_grad():
        out, _ = m(x.to(cuda))
    d = (out.cpu().float() - ref.float()).abs()
    # bf16 projections (cuBLAS vs CPU) perturb routing near ties; the layer output stays within the
    # bf16 attention tolerance on average and close everywhere
    assert (d.sum() / ref.float().abs().sum()).item() < 2e-2
    assert d.max().item() < 0.25
