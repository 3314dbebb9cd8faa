"""Sharded prefill (query chunks split across ranks, K/V + summaries all-gathered) equals the
single-device module forward.  The ranks are emulated in one process: every rank's local phase
runs, the send buffers are concatenated (what the all-gather produces), then every rank's global
phase runs — no kernel waits on another rank."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _module(dev, d_model=1024, nhead=8, kv_heads=2, head_dim=128, seed=0):
    from hierarchicalglobalattention_b200 import HierarchicalGlobalAttentionRouted
    torch.manual_seed(seed)
    m = HierarchicalGlobalAttentionRouted(d_model=d_model, nhead=nhead, kv_heads=kv_heads, head_dim=head_dim,
                                          qk_norm=True, theta=1e6, chunk_size=64, group_size=16, keep_first=2,
                                          keep_last=8, topk_chunks=16, topk_groups=64)
    with torch.no_grad():
        for n, p in m.named_parameters():
            p.normal_(1.0, 0.1) if "norm" in n else p.normal_(0.0, 0.02)
    return m.to(device=dev, dtype=torch.bfloat16).eval()


def emulate(m, x, S, W):
    from hierarchicalglobalattention_b200.shard import ShardedPrefill, prefill_partition
    parts = prefill_partition(S, 64, W)
    shards = [ShardedPrefill(W, r, exchange=lambda s: s) for r in range(W)]
    states, sends = [], []
    for r, (lo, hi) in enumerate(parts):
        st, send = shards[r].local_phase(m, x[:, lo * 64:min(S, hi * 64)], S)
        states.append(st)
        sends.append(send.clone())
    lay = states[0]["lay"]
    recv = torch.stack(sends)
    rs, rk = recv[:, :lay.sum_numel].contiguous().view(-1), recv[:, lay.sum_numel:].contiguous().view(-1)
    return [shards[r].global_phase(m, states[r], rs, rk) for r in range(W)]


@pytest.mark.parametrize("S,W", [(1000, 3), (4096, 8), (2048, 2), (200, 8)])
def test_sharded_prefill_equals_single_device(cuda, S, W):
    m = _module(cuda)
    x = torch.randn(1, S, m.d_model, device=cuda, dtype=torch.bfloat16, generator=torch.Generator(cuda).manual_seed(1))
    with torch.no_grad():
        ref, _ = m(x)
        outs = emulate(m, x, S, W)
    out = torch.cat([o for o in outs if o is not None], dim=1)
    assert out.shape == ref.shape
    d = (out.float() - ref.float()).abs()
    # the only difference is the QKV GEMM over a row subset (cuBLAS may pick another tiling), which
    # can move a score across a bf16 rounding boundary: nearly all rows are identical
    assert (d.amax(-1) == 0).float().mean() > 0.9
    assert d.max() < 5e-2
