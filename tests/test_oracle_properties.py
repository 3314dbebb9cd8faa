"""Properties of the CPU oracle that hold whatever the routing decides, after the reference's own
router tests (ExistingModelFineTuning/KvRouter/Tests/test_router.py:37-82): with every chunk kept
token-level and no routing the incremental path is dense causal attention, and no query row ever
depends on a later token."""
import pytest
import torch
import torch.nn.functional as F

from oracle import hga_oracle as O


def _inputs(p, B, S, seed, dtype=torch.float32):
    g = torch.Generator().manual_seed(seed)
    H, KVH, Dh = p.nhead, p.kv_heads, p.head_dim
    q = torch.randn(B, H, S, Dh, generator=g).to(dtype)
    k_raw = torch.randn(B, KVH, S, Dh, generator=g).to(dtype)
    v = torch.randn(B, KVH, S, Dh, generator=g).to(dtype)
    cos, sin = O.module_rotary(p.theta, Dh, S)
    half = Dh // 2
    kf = k_raw.float()
    k_rope = (kf * cos + torch.cat((-kf[..., half:], kf[..., :half]), -1) * sin).to(dtype)
    return q, k_rope, k_raw, v


@pytest.mark.parametrize("block", [1, 3, 8])
def test_incremental_path_with_everything_kept_is_dense_causal(block):
    """keep_first covering every chunk, no routing: the decode path == causal SDPA (28 tokens = 3
    closed chunks and a partial one, as in the reference's test)."""
    p = O.OracleParams(nhead=8, kv_heads=4, head_dim=16, chunk_size=8, group_size=4, topk_chunks=0,
                       topk_groups=0, keep_first=999, keep_last=0, theta=1e4)
    B, S = 2, 28
    q, k_rope, k_raw, v = _inputs(p, B, S, seed=1)
    out, _ = O.decode_sequence(p, q, k_rope, k_raw, v, block)
    ref = F.scaled_dot_product_attention(q, k_rope.repeat_interleave(p.rep, 1), v.repeat_interleave(p.rep, 1),
                                         is_causal=True)
    assert (out - ref).abs().max().item() < 1e-5


@pytest.mark.parametrize("path", ["incremental", "prefill"])
def test_no_row_depends_on_a_later_token(path):
    """Perturbing every token from position t on leaves the outputs of rows < t unchanged, on the
    routed (sparse) configuration.  t starts a chunk (and so a decode block): inside one block or
    query chunk the routing pools over all its rows (chunk_router.py:222-232, vectorized.py:99-140),
    so a later row may change which chunk an earlier row of the same unit sees, by design."""
    p = O.OracleParams(nhead=4, kv_heads=2, head_dim=16, chunk_size=8, group_size=4, topk_chunks=2,
                       topk_groups=4, keep_first=1, keep_last=1, theta=1e4)
    B, S, t = 1, 72, 40
    q, k_rope, k_raw, v = _inputs(p, B, S, seed=2)
    q2, k_rope2, k_raw2, v2 = (x.clone() for x in (q, k_rope, k_raw, v))
    g = torch.Generator().manual_seed(9)
    for x in (q2, k_rope2, k_raw2, v2):
        x[:, :, t:] = torch.randn(x[:, :, t:].shape, generator=g)

    def run(q_, kr_, kw_, v_):
        if path == "incremental":
            return O.decode_sequence(p, q_, kr_, kw_, v_, 5)[0]
        ck, gk, _ = O.summaries_prefill(p, kw_, kr_, v_, *O.module_rotary(p.theta, p.head_dim, S))
        route = O.route_prefill(p, q_, ck, gk, S)
        return O.attend_prefill(p, q_, kr_, v_, route, S)

    a, b = run(q, k_rope, k_raw, v), run(q2, k_rope2, k_raw2, v2)
    assert torch.isfinite(a).all() and torch.isfinite(b).all()
    assert torch.equal(a[:, :, :t], b[:, :, :t])
    assert not torch.equal(a[:, :, t:], b[:, :, t:])
