"""Routed attention for pretrained Qwen3 / Qwen3-MoE models on the B200 kernels.

Drop-in for the reference's Qwen3 patch
(ExistingModelFineTuning/Qwen3LongContext/qwen_routed_attention.py:94-399):
``replace_qwen_attention_with_router(model, ...)`` swaps every decoder layer's ``self_attn`` for a
``QwenRoutedAttention`` that keeps the original module as the child ``orig`` and reuses its
q/k/v/o projections and q/k RMSNorms by reference (no new parameters);
``restore_original_attention(model)`` puts the originals back.  Same keyword arguments, defaults,
forward signature and return value ``(out, None)``, and one router/store per model attached to the
``past_key_values`` object (``_kv_router``).

The arithmetic follows the HF layers the reference calls: Qwen3 RMSNorm (fp32 normalisation,
rounded to the model dtype before the weight product) and ``apply_rotary_pos_emb`` on the model's
own ``position_embeddings`` (model-dtype products), fused into one prologue kernel after a single
concatenated QKV projection GEMM.  RoPE theta is read from ``config.rope_parameters`` (transformers
5) or ``config.rope_theta`` (older releases), default 1e6.

Dual Chunk Attention (``dca_chunk > 0``, qwen_routed_attention.py:210-283): keys stored roped at
their intra-chunk position ``pos % dca_chunk``, routed with intra-roped queries through the
incremental path, attended by the DCA decode kernel (three fp32 ropings of each query chosen per
key by DCA chunk).  Not carried over: the file-system cache tier (``cache_location="fs"``), which
raises.
"""
from __future__ import annotations

from typing import Any, Optional, Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F

from .config import ChunkPlacementPolicy, RouterConfig
from . import ops
from .module import routed_attention
from .router import ChunkRouter
from .store import VramKVCacheStore


def rope_theta_of(config: Any, default: float = 1_000_000.0) -> float:
    """RoPE base of a HF config: ``rope_parameters["rope_theta"]`` (transformers >= 5) or
    ``rope_theta``."""
    rp = getattr(config, "rope_parameters", None)
    if isinstance(rp, dict) and rp.get("rope_theta") is not None:
        return float(rp["rope_theta"])
    try:
        v = getattr(config, "rope_theta")
    except AttributeError:
        v = None
    return float(v) if v is not None else float(default)


def dca_rotate(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """rotate-half RoPE in x's dtype (qwen_routed_attention.py:84-88; HF apply_rotary_pos_emb)."""
    half = x.shape[-1] // 2
    return x * cos + torch.cat((-x[..., half:], x[..., :half]), dim=-1) * sin


def dca_forward(router: ChunkRouter, layer: int, q: torch.Tensor, k_raw: torch.Tensor, v: torch.Tensor,
                start_pos: int, dca_chunk: int, dca_ceil: int, theta: float) -> torch.Tensor:
    """Dual Chunk Attention of one forward call on normalised, pre-RoPE tensors
    (QwenRoutedAttention._dca_forward, qwen_routed_attention.py:210-245): q [B,H,S,Dh], k_raw / v
    [B,KVH,S,Dh] at positions [start_pos, start_pos + S).  Keys are roped at pos % dca_chunk (the
    store keeps them so), routed with equally roped queries through the incremental path, and
    each chunk piece is attended by the DCA kernel before the next is routed.  Returns the heads
    [B,H,S,Dh]."""
    B, H, S, Dh = q.shape
    C = router.cfg.chunk_size
    pos = torch.arange(start_pos, start_pos + S, device=q.device)
    tc, ts = ops.dca_rope_table(dca_ceil, Dh, theta, q.device)
    cos, sin = tc[pos % dca_chunk].to(q.dtype), ts[pos % dca_chunk].to(q.dtype)
    k_dca = dca_rotate(k_raw, cos, sin)
    q_sel = dca_rotate(q, cos, sin)
    out = torch.empty_like(q)
    p, done = start_pos, 0
    while done < S:
        take = min(C - (p % C), S - done)
        sl = slice(done, done + take)
        rk = router.decode_block(layer, q_sel[:, :, sl], k_dca[:, :, sl].contiguous(), k_raw[:, :, sl].contiguous(),
                                 v[:, :, sl].contiguous(), p, return_positions=True)
        out[:, :, sl] = rk.attend_dca(q[:, :, sl], pos[sl], dca_chunk, dca_ceil, theta)
        p += take
        done += take
    return out


class QwenRoutedAttention(nn.Module):
    """Replacement for ``Qwen3MoeAttention`` / ``Qwen3Attention`` routing through a shared
    ``ChunkRouter``; adds no parameters."""

    def __init__(self, orig: nn.Module, config: Any, *, chunk_size: int = 64, group_size: int = 16,
                 keep_first: int = 2, keep_last: int = 2, topk_chunks: int = 8, topk_groups: int = 32,
                 cache_location: str = "vram", vram_cache_chunks: int = 256, vram_summary_chunks: int = 4096,
                 vram_cache_reserve_gb: float = 1.5, ram_budget_gb: float = 12.0,
                 fs_cache_dir: Optional[str] = None, dca_chunk: int = 0, dca_local: int = 0) -> None:
        super().__init__()
        if cache_location not in ("vram", "ram"):
            raise NotImplementedError(f"cache_location={cache_location!r}: the B200 path provides 'vram' and 'ram'")
        self.orig = orig
        self.layer_idx = int(getattr(orig, "layer_idx", 0))
        self.num_heads = int(config.num_attention_heads)
        self.num_kv_heads = int(getattr(config, "num_key_value_heads", None) or self.num_heads)
        hd = getattr(config, "head_dim", None)
        self.head_dim = int(hd) if hd else config.hidden_size // self.num_heads
        self.num_layers = int(getattr(config, "num_hidden_layers", 0))
        self.chunk_size = chunk_size
        self.cache_location = cache_location
        self.vram_cache_chunks = vram_cache_chunks
        self.vram_summary_chunks = vram_summary_chunks
        self.vram_cache_reserve_gb = vram_cache_reserve_gb
        self.ram_budget_gb = ram_budget_gb
        self.fs_cache_dir = fs_cache_dir
        if dca_chunk > 0 and dca_chunk % chunk_size != 0:
            # a routing chunk must lie inside one DCA chunk (qwen_routed_attention.py:137-141)
            raise ValueError(f"dca_chunk ({dca_chunk}) must be a multiple of chunk_size ({chunk_size})")
        self.dca_chunk = max(0, int(dca_chunk))
        # local window added to the chunk length: default a fifth of the chunk (at least 1)
        self.dca_local = (int(dca_local) if dca_local > 0 else max(1, self.dca_chunk // 5)) if self.dca_chunk else 0
        self.dca_ceil = self.dca_chunk + self.dca_local
        self._cfg = RouterConfig(nhead=self.num_heads, kv_heads=self.num_kv_heads, head_dim=self.head_dim,
                                 chunk_size=chunk_size, group_size=group_size, topk_chunks=topk_chunks,
                                 topk_groups=topk_groups, theta=rope_theta_of(config))
        self._policy = ChunkPlacementPolicy(keep_last=keep_last, keep_first=keep_first, first_token_level=True)
        self._qkv_cache = None

    # ------------------------------------------------------------------------------------------
    def _qkv(self, x: torch.Tensor) -> torch.Tensor:
        """[B,S,(H+2KVH)*Dh] projection output: one GEMM over the concatenated weights when the
        projections are plain ``nn.Linear`` layers, else the three modules' outputs concatenated."""
        o = self.orig
        projs = (o.q_proj, o.k_proj, o.v_proj)
        if all(type(m) is nn.Linear for m in projs):
            ps = tuple(m.weight for m in projs) + tuple(m.bias for m in projs)
            key = tuple((t.data_ptr(), t._version, t.dtype) if t is not None else None for t in ps)
            if self._qkv_cache is None or self._qkv_cache[0] != key:
                w = torch.cat([m.weight for m in projs], dim=0).detach()
                b = None
                if any(m.bias is not None for m in projs):
                    b = torch.cat([m.bias if m.bias is not None else
                                   torch.zeros(m.out_features, device=w.device, dtype=w.dtype) for m in projs]).detach()
                self._qkv_cache = (key, w, b)
            return F.linear(x, self._qkv_cache[1], self._qkv_cache[2])
        return torch.cat([m(x) for m in projs], dim=-1).contiguous()

    def forward(self, hidden_states: torch.Tensor, position_embeddings: Tuple[torch.Tensor, torch.Tensor],
                attention_mask: Optional[torch.Tensor] = None, past_key_values: Any = None,
                cache_position: Optional[torch.Tensor] = None, **kw: Any) -> Tuple[torch.Tensor, None]:
        o = self.orig
        x = hidden_states
        B, S, _ = x.shape
        H, Dh = self.num_heads, self.head_dim
        start_pos = 0
        if cache_position is not None and cache_position.numel() > 0:
            start_pos = int(cache_position.reshape(-1)[0].item())
        else:
            pos_ids = kw.get("position_ids", None)
            if pos_ids is not None and pos_ids.numel() > 0:
                start_pos = int(pos_ids.reshape(-1)[0].item())
        router = self._get_router(past_key_values, B, x.dtype, x.device)
        if self.layer_idx == 0 and start_pos == 0:
            router.reset()
        if self.dca_chunk > 0:
            return self._dca_forward(x, start_pos, router), None
        cos, sin = position_embeddings
        # rows of the model's own table (batch row 0: every sequence of the batch is at the same positions)
        cos = cos.reshape(-1, S, Dh)[0].to(x.dtype).contiguous()
        sin = sin.reshape(-1, S, Dh)[0].to(x.dtype).contiguous()
        qkv = self._qkv(x)
        hp = self._cfg.hga_params(self._policy, B, x.dtype)
        qn = o.q_norm.weight.detach().to(x.dtype).contiguous()
        kn = o.k_norm.weight.detach().to(x.dtype).contiguous()
        eps = float(getattr(o.q_norm, "variance_epsilon", getattr(o.q_norm, "eps", 1e-6)))
        out_heads = routed_attention(router, self.layer_idx, hp, qkv, cos, sin, start_pos, start_pos, qn, kn, eps,
                                     norm_mode=1, rope_mode=1, round_table=False)
        return o.o_proj(out_heads.view(B, S, H * Dh)), None

    # ------------------------------------------------------------------------------------------
    def _dca_forward(self, x: torch.Tensor, start_pos: int, router: ChunkRouter) -> torch.Tensor:
        """Dual Chunk Attention (QwenRoutedAttention._dca_forward / _dca_attend,
        qwen_routed_attention.py:210-283).  The prologue kernel runs twice on the fused projection:
        with the model-dtype RoPE rows of the intra-chunk positions (selection queries, stored
        keys, pre-RoPE keys, values) and with an identity table (cos 1, sin 0: the normalised
        queries unchanged, which the DCA attention ropes three ways itself).  Blocks go through
        the incremental router chunk by chunk, each attended before the next is routed."""
        o = self.orig
        B, S, _ = x.shape
        H, Dh, C, L_c = self.num_heads, self.head_dim, self.chunk_size, self.dca_chunk
        theta = self._cfg.theta
        qkv = self._qkv(x)
        hp = self._cfg.hga_params(self._policy, B, x.dtype)
        qn = o.q_norm.weight.detach().to(x.dtype).contiguous()
        kn = o.k_norm.weight.detach().to(x.dtype).contiguous()
        eps = float(getattr(o.q_norm, "variance_epsilon", getattr(o.q_norm, "eps", 1e-6)))
        pos = torch.arange(start_pos, start_pos + S, device=x.device)
        tc, ts = ops.dca_rope_table(self.dca_ceil, Dh, theta, x.device)
        cos, sin = tc[pos % L_c].to(x.dtype), ts[pos % L_c].to(x.dtype)
        q_sel, k_raw, k_dca, v = ops.qkv_prologue(hp, qkv, cos, sin, q_norm_w=qn, k_norm_w=kn, eps=eps, norm_mode=1,
                                                  rope_mode=1, rot_row0=start_pos, pos0=start_pos)
        one, zero = torch.ones_like(cos), torch.zeros_like(sin)
        q_raw = ops.qkv_prologue(hp, qkv, one, zero, q_norm_w=qn, k_norm_w=kn, eps=eps, norm_mode=1, rope_mode=1,
                                 rot_row0=start_pos, pos0=start_pos)[0]
        out_heads = torch.empty(B, S, H, Dh, device=x.device, dtype=x.dtype)
        p, done = start_pos, 0
        while done < S:
            take = min(C - (p % C), S - done)
            sl = slice(done, done + take)
            rk = router.decode_block(self.layer_idx, q_sel[:, :, sl], k_dca[:, :, sl], k_raw[:, :, sl], v[:, :, sl], p,
                                     return_positions=True)
            out_heads[:, sl] = rk.attend_dca(q_raw[:, :, sl], pos[sl], L_c, self.dca_ceil, theta).transpose(1, 2)
            p += take
            done += take
        return o.o_proj(out_heads.view(B, S, H * Dh))

    # ------------------------------------------------------------------------------------------
    def _make_store(self, B: int, dtype: torch.dtype, device: torch.device):
        kwargs = dict(compute_device=device, policy=self._policy, kv_heads=self.num_kv_heads, head_dim=self.head_dim,
                      chunk_size=self.chunk_size, groups_per_chunk=self._cfg.groups_per_chunk, batch_size=B,
                      dtype=dtype)
        if self.cache_location == "vram":
            return VramKVCacheStore(**kwargs)
        from .store_ram import RamKVCacheStore
        return RamKVCacheStore(pin_memory=True, vram_cache_chunks=self.vram_cache_chunks,
                               vram_summary_chunks=self.vram_summary_chunks, num_layers=self.num_layers,
                               vram_cache_reserve_gb=self.vram_cache_reserve_gb, **kwargs)

    def _get_router(self, pkv: Any, B: int, dtype: torch.dtype, device: torch.device) -> ChunkRouter:
        """One router/store shared by all layers, attached to the ``past_key_values`` object."""
        holder = pkv if pkv is not None else self
        router = getattr(holder, "_kv_router", None)
        if router is None:
            router = ChunkRouter(self._cfg, self._make_store(B, dtype, device))
            setattr(holder, "_kv_router", router)
        return router


def _attention_layers(model: nn.Module):
    layers = getattr(getattr(model, "model", None), "layers", None)
    if layers is None:
        raise RuntimeError("model.model.layers not found")
    for layer in layers:
        if hasattr(layer, "self_attn"):
            yield layer


def restore_original_attention(model: nn.Module) -> int:
    """Undo ``replace_qwen_attention_with_router``; returns the number of layers restored."""
    n = 0
    for layer in _attention_layers(model):
        if isinstance(layer.self_attn, QwenRoutedAttention):
            layer.self_attn = layer.self_attn.orig
            n += 1
    return n


def replace_qwen_attention_with_router(model: nn.Module, *, keep_first: int = 2, keep_last: int = 2,
                                       topk_chunks: int = 8, topk_groups: int = 32, chunk_size: int = 64,
                                       group_size: int = 16, cache_location: str = "vram",
                                       vram_cache_chunks: int = 256, vram_summary_chunks: int = 4096,
                                       vram_cache_reserve_gb: float = 1.5, ram_budget_gb: float = 12.0,
                                       fs_cache_dir: Optional[str] = None, dca_chunk: int = 0,
                                       dca_local: int = 0) -> int:
    """Replace every decoder layer's ``self_attn`` with a ``QwenRoutedAttention`` (idempotent:
    earlier replacements are undone first).  Returns the number of layers replaced."""
    restore_original_attention(model)
    config = model.config
    count = 0
    for layer in _attention_layers(model):
        layer.self_attn = QwenRoutedAttention(
            layer.self_attn, config, chunk_size=chunk_size, group_size=group_size, keep_first=keep_first,
            keep_last=keep_last, topk_chunks=topk_chunks, topk_groups=topk_groups, cache_location=cache_location,
            vram_cache_chunks=vram_cache_chunks, vram_summary_chunks=vram_summary_chunks,
            vram_cache_reserve_gb=vram_cache_reserve_gb, ram_budget_gb=ram_budget_gb, fs_cache_dir=fs_cache_dir,
            dca_chunk=dca_chunk, dca_local=dca_local)
        count += 1
    return count


__all__ = ["QwenRoutedAttention", "replace_qwen_attention_with_router", "restore_original_attention", "rope_theta_of"]
