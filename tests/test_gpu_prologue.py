"""The fused q/k RMSNorm + RoPE + layout prologue (hga_qkv_prologue) against a torch fp32 / model-dtype
restatement of both norm modes (the routed module's RMSNorm and HF Qwen3's) and both RoPE modes."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _ref(qkv, H, KVH, Dh, qw, kw, eps, norm_mode, rope_mode, cos, sin, pos0, rot_row0):
    B, S, _ = qkv.shape
    dt = qkv.dtype
    x = qkv[..., :(H + 2 * KVH) * Dh].reshape(B, S, H + 2 * KVH, Dh)
    q, k, v = x[:, :, :H], x[:, :, H:H + KVH], x[:, :, H + KVH:]

    def norm(t, w):
        if w is None:
            return t
        tf = t.float()
        rs = torch.rsqrt(tf.pow(2).mean(-1, keepdim=True) + eps)
        if norm_mode == 0:
            return (w.float() * tf * rs).to(dt)
        return w * (tf * rs).to(dt)

    q, k = norm(q, qw), norm(k, kw)
    c = cos[pos0 - rot_row0:pos0 - rot_row0 + S].view(1, S, 1, Dh)
    s_ = sin[pos0 - rot_row0:pos0 - rot_row0 + S].view(1, S, 1, Dh)

    def rope(t):
        rot = torch.cat((-t[..., Dh // 2:], t[..., :Dh // 2]), -1)
        if rope_mode == 0:
            return (t.float() * c + rot.float() * s_).to(dt)
        return t * c + rot * s_

    return rope(q), k, rope(k), v


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("Dh", [128, 64, 32])
@pytest.mark.parametrize("norm_mode,rope_mode", [(0, 0), (1, 1)])
def test_prologue_matches_torch(cuda, dtype, Dh, norm_mode, rope_mode):
    from hierarchicalglobalattention_b200 import _lib, ops
    B, S, H, KVH = 2, 100, 4, 2
    g = torch.Generator(device=cuda).manual_seed(Dh + norm_mode)
    qkv = torch.randn(B, S, (H + 2 * KVH) * Dh, device=cuda, generator=g).to(dtype)
    qw = (1 + 0.1 * torch.randn(Dh, device=cuda, generator=g)).to(dtype)
    kw = (1 + 0.1 * torch.randn(Dh, device=cuda, generator=g)).to(dtype)
    pos0, rot_row0 = 37, 5
    half = Dh // 2
    inv = 1.0 / (1e4 ** (torch.arange(half, dtype=torch.float32) / half))
    f = torch.arange(rot_row0, pos0 + S, dtype=torch.float32)[:, None] * inv
    emb = torch.cat((f, f), -1)
    cos, sin = emb.cos().to(cuda), emb.sin().to(cuda)
    if rope_mode == 1:
        cos, sin = cos.to(dtype), sin.to(dtype)
    hp = _lib.make_params(batch=B, nhead=H, kv_heads=KVH, head_dim=Dh, chunk_size=64, group_size=16, topk_chunks=4,
                          topk_groups=8, keep_first=1, keep_last=1, theta=1e4, dtype=dtype)
    q, kr, kp, v = ops.qkv_prologue(hp, qkv, cos, sin, q_norm_w=qw, k_norm_w=kw, eps=1e-6, norm_mode=norm_mode,
                                    rope_mode=rope_mode, rot_row0=rot_row0, pos0=pos0)
    rq, rkr, rkp, rv = _ref(qkv, H, KVH, Dh, qw, kw, 1e-6, norm_mode, rope_mode, cos, sin, pos0, rot_row0)
    tol = dict(atol=1e-5, rtol=1e-5) if dtype == torch.float32 else dict(atol=2e-2, rtol=1e-2)
    torch.testing.assert_close(q.transpose(1, 2).float(), rq.float(), **tol)
    torch.testing.assert_close(kr.float(), rkr.transpose(1, 2).float(), **tol)
    torch.testing.assert_close(kp.float(), rkp.transpose(1, 2).float(), **tol)
    assert torch.equal(v, rv.transpose(1, 2).contiguous())
    if dtype == torch.bfloat16:   # nearly every element lands on the same bf16 value
        assert (q.transpose(1, 2) == rq).float().mean() > 0.97
