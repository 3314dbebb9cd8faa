"""torch.ops.hga.*: the operators are registered with schemas, and their fake implementations
give the C entry points' output shapes on meta tensors (no GPU, no kernel)."""
import torch

import hierarchicalglobalattention_b200 as hga
from hierarchicalglobalattention_b200 import _lib, torch_ops


def _p():
    return _lib.make_params(batch=2, nhead=8, kv_heads=2, head_dim=64, chunk_size=64, group_size=16, topk_chunks=4,
                            topk_groups=8, keep_first=1, keep_last=2, theta=1e4, dtype=torch.bfloat16)


def test_ops_are_registered():
    for name in ("summaries", "route_prefill", "attend_prefill", "route_decode", "attend_decode", "attend_decode_dca", "gather_h2d"):
        assert hasattr(torch.ops.hga, name), name
    assert "Tensor(a3!) bank_k" in str(torch.ops.hga.gather_h2d.default._schema) or "bank_k" in str(
        torch.ops.hga.gather_h2d.default._schema)


def test_fake_shapes_on_meta():
    pi, pf = torch_ops.params_lists(_p())
    m = dict(device="meta", dtype=torch.bfloat16)
    B, H, KVH, S, Dh = 2, 8, 2, 1000, 64
    k = torch.empty(B, KVH, S, Dh, **m)
    cos = torch.empty(S, Dh, device="meta")
    ck, gk, gv = torch.ops.hga.summaries(pi, pf, k, k, k, cos, cos, True)
    assert ck.shape == (B, KVH, 16, Dh) and gk.shape == (B, KVH, 16, 4, Dh) and gv.shape == gk.shape
    q = torch.empty(B, H, S, Dh, **m)
    sc, st, og, ot = torch.ops.hga.route_prefill(pi, pf, q, ck, gk)
    assert sc.shape == (B, H, 16, 4) and og.shape == (B, H, 16, 8) and og.dtype == torch.int32
    out = torch.ops.hga.attend_prefill(pi, pf, q, k, k, og, ot)
    assert out.shape == (B, S, H, Dh)
    qd = torch.empty(B, H, 1, Dh, **m)
    pos = torch.empty(B, dtype=torch.int32, device="meta")
    mc, mt, og2, ot2 = torch.ops.hga.route_decode(pi, pf, qd, pos, ck, gk, 10)
    assert mc.shape == (B, H, 4) and og2.shape == (B, H, 8)
    assert torch.ops.hga.attend_decode(pi, pf, qd, pos, k, k, 0, None, None, og2, ot2).shape == qd.shape
    assert torch.ops.hga.attend_decode_dca(pi, pf, qd, pos, k, k, 0, None, None, og2, ot2, None, 256, 300,
                                           1e6).shape == qd.shape
    assert hga.ops is not None
