"""``HierarchicalGlobalAttentionRouted`` — drop-in for the reference module
(ExistingModelFineTuning/HierarchicalGlobalAttentionRouted.py:70-250).

Same constructor, parameter names (``q_proj/k_proj/v_proj/o_proj/q_norm/k_norm``, so reference
state_dicts load unchanged), forward signature, return value ``(out, {})`` and router placement
(``past_key_value._kv_router`` or the module itself).  The forward runs:

  one fused QKV projection GEMM (cuBLAS via torch)  ->  hga_qkv_prologue (RMSNorm + RoPE + store
  layout)  ->  ChunkRouter (summary builder, two-level router / incremental decode kernels)  ->
  working-set attention kernel writing [B,S,H,Dh]  ->  o_proj GEMM.
"""
from __future__ import annotations

from typing import Any, Optional, Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import ops
from .config import ChunkPlacementPolicy, RouterConfig
from .router import ChunkRouter
from .store import VramKVCacheStore


def routed_attention(router: ChunkRouter, layer: int, hp, qkv: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor,
                     rot_row0: int, start_pos: int, q_norm_w: Optional[torch.Tensor], k_norm_w: Optional[torch.Tensor],
                     eps: float, *, norm_mode: int, rope_mode: int, round_table: bool) -> torch.Tensor:
    """Attention core shared by the routed module and the Qwen3 wrapper: q/k RMSNorm + RoPE
    prologue on the fused projection output ``qkv`` [B,S,(H+2KVH)*Dh], routing through ``router``
    and the routed attention kernels.  Returns the heads' output [B,S,H,Dh] (o_proj input layout).

    ``cos``/``sin`` [R, Dh] hold the rotary rows of positions [rot_row0, rot_row0 + R): fp32 for
    rope_mode 0, the model dtype for rope_mode 1.  A fresh multi-chunk prefill into a VRAM store
    writes K/V straight into the store's token rows (no seed copy)."""
    B, S, _ = qkv.shape
    H, KVH, Dh, C = hp.nhead, hp.kv_heads, hp.head_dim, hp.chunk_size
    multi_chunk = start_pos // C != (start_pos + S - 1) // C
    store = router.store
    kv_out = None
    if start_pos == 0 and multi_chunk and not getattr(store, "cold_on_host", False):
        # k_raw gets a scratch buffer with the token rows' capacity
        st = store.ensure_capacity(layer, max(S // C, 1), S)
        kraw_buf = torch.empty(B, KVH, st.tcap, Dh, device=qkv.device, dtype=qkv.dtype)
        kv_out = (kraw_buf, st.token_k, st.token_v)
    q_rope, k_raw, k_rope, v = ops.qkv_prologue(hp, qkv, cos, sin, q_norm_w=q_norm_w, k_norm_w=k_norm_w, eps=eps,
                                                norm_mode=norm_mode, rope_mode=rope_mode, rot_row0=rot_row0,
                                                pos0=start_pos, kv_out=kv_out, kv_row0=0)
    out_heads = torch.empty(B, S, H, Dh, device=qkv.device, dtype=qkv.dtype)
    r0 = start_pos - rot_row0
    segments = router.route_query_block(layer, q_rope, k_rope, k_raw, v, start_pos,
                                        cos=cos[r0:r0 + S].view(1, 1, S, Dh), sin=sin[r0:r0 + S].view(1, 1, S, Dh),
                                        _round_table=round_table, _out=out_heads)
    for routed, lo, hi in segments:
        if routed.chunked and lo == 0 and hi == S:
            routed.attend(q_rope, use_summaries=False)
        else:
            out_heads[:, lo:hi] = routed.attend(q_rope[:, :, lo:hi], use_summaries=False).transpose(1, 2)
    return out_heads


class RMSNorm(nn.Module):
    """RMSNorm with the reference's parameter name and fp32 arithmetic (HierarchicalGlobalAttentionRouted.py:56-67)."""

    def __init__(self, dim: int, eps: float = 1e-6) -> None:
        super().__init__()
        self.weight = nn.Parameter(torch.ones(dim))
        self.eps = eps

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        xf = x.float()
        return (self.weight.float() * xf * torch.rsqrt(xf.pow(2).mean(dim=-1, keepdim=True) + self.eps)).to(x.dtype)


class HierarchicalGlobalAttentionRouted(nn.Module):
    """Chunk-routed causal self-attention backed by the B200 kernels."""

    def __init__(self, d_model: int, nhead: int = 16, kv_heads: int = 8, dropout: float = 0.0,
                 use_bias_q: bool = False, use_bias_k: bool = False, use_bias_v: bool = False,
                 use_bias_o: bool = False, causal: bool = True, chunk_size: int = 64, group_size: int = 16,
                 topk_chunks: int = 20, topk_groups: int = 32, keep_first: int = 1, keep_last: int = 2,
                 head_dim: Optional[int] = None, qk_norm: bool = False, norm_eps: float = 1e-6,
                 theta: float = 1_000_000.0, layer_idx: int = 0, cache_location: str = "vram",
                 num_layers: int = 0, **kwargs: Any) -> None:
        super().__init__()
        assert nhead % kv_heads == 0
        head_dim = d_model // nhead if head_dim is None else head_dim
        self.d_model, self.nhead, self.kv_heads, self.head_dim = d_model, nhead, kv_heads, head_dim
        self.theta = float(theta)
        self.dropout_p = dropout
        self.layer_idx = layer_idx
        self.cache_location = cache_location
        self.num_layers = num_layers
        self.chunk_size = chunk_size
        self.norm_eps = norm_eps
        self.q_proj = nn.Linear(d_model, nhead * head_dim, bias=use_bias_q)
        self.k_proj = nn.Linear(d_model, kv_heads * head_dim, bias=use_bias_k)
        self.v_proj = nn.Linear(d_model, kv_heads * head_dim, bias=use_bias_v)
        self.o_proj = nn.Linear(nhead * head_dim, d_model, bias=use_bias_o)
        if qk_norm:
            self.q_norm: nn.Module = RMSNorm(head_dim, eps=norm_eps)
            self.k_norm: nn.Module = RMSNorm(head_dim, eps=norm_eps)
        else:
            self.q_norm = nn.Identity()
            self.k_norm = nn.Identity()
        self._cfg = RouterConfig(nhead=nhead, kv_heads=kv_heads, head_dim=head_dim, chunk_size=chunk_size,
                                 group_size=group_size, topk_chunks=topk_chunks, topk_groups=topk_groups,
                                 theta=theta)
        self._policy = ChunkPlacementPolicy(keep_first=keep_first, keep_last=keep_last, first_token_level=True)
        self._qkv_cache: Optional[Tuple] = None
        self._rot: Optional[Tuple[torch.Tensor, torch.Tensor]] = None

    # ------------------------------------------------------------------------------------------
    def _fused_qkv(self):
        """Concatenated [q;k;v] projection weight (and bias), rebuilt when any parameter changes."""
        ps = (self.q_proj.weight, self.k_proj.weight, self.v_proj.weight,
              self.q_proj.bias, self.k_proj.bias, self.v_proj.bias)
        key = tuple((p.data_ptr(), p._version, p.dtype) if p is not None else None for p in ps)
        if self._qkv_cache is None or self._qkv_cache[0] != key:
            w = torch.cat([self.q_proj.weight, self.k_proj.weight, self.v_proj.weight], dim=0).detach()
            b = None
            if any(p is not None for p in ps[3:]):
                b = torch.cat([p if p is not None else torch.zeros(q.weight.shape[0], device=w.device, dtype=w.dtype)
                               for p, q in zip(ps[3:], (self.q_proj, self.k_proj, self.v_proj))]).detach()
            self._qkv_cache = (key, w, b)
        return self._qkv_cache[1], self._qkv_cache[2]

    def _own_rotary(self, n: int, device) -> Tuple[torch.Tensor, torch.Tensor]:
        """fp32 cos/sin [n, Dh] (HierarchicalGlobalAttentionRouted.py:209-217), cached."""
        if self._rot is None or self._rot[0].shape[0] < n or self._rot[0].device != torch.device(device):
            m = max(n, 2 * self._rot[0].shape[0] if self._rot is not None else n)
            half = self.head_dim // 2
            inv = 1.0 / (self.theta ** (torch.arange(0, half, device=device, dtype=torch.float32) / half))
            t = torch.arange(m, device=device, dtype=torch.float32)
            f = torch.einsum("i,j->ij", t, inv)
            emb = torch.cat((f, f), dim=-1)
            self._rot = (emb.cos(), emb.sin())
        return self._rot

    def _rotary_for(self, position_embeddings, start_pos: int, S: int, device):
        if position_embeddings is not None:
            cos, sin = position_embeddings
            cos = cos.to(device=device, dtype=torch.float32).reshape(-1, self.head_dim)[-S:]
            sin = sin.to(device=device, dtype=torch.float32).reshape(-1, self.head_dim)[-S:]
            return cos.contiguous(), sin.contiguous(), start_pos
        cos, sin = self._own_rotary(start_pos + S, device)
        return cos, sin, 0

    def _make_store(self, B: int, dtype, device):
        kwargs = dict(compute_device=device, policy=self._policy, kv_heads=self.kv_heads, head_dim=self.head_dim,
                      chunk_size=self.chunk_size, groups_per_chunk=self._cfg.groups_per_chunk, batch_size=B,
                      dtype=dtype)
        if self.cache_location == "vram":
            return VramKVCacheStore(**kwargs)
        from .store_ram import RamKVCacheStore
        return RamKVCacheStore(pin_memory=True, num_layers=self.num_layers, **kwargs)

    def _get_router(self, pkv: Any, B: int, dtype, device) -> ChunkRouter:
        holder = pkv if pkv is not None else self
        router = getattr(holder, "_kv_router", None)
        if router is None:
            router = ChunkRouter(self._cfg, self._make_store(B, dtype, device))
            setattr(holder, "_kv_router", router)
        return router

    # ------------------------------------------------------------------------------------------
    def forward(self, hidden_states: Optional[torch.Tensor] = None,
                position_embeddings: Optional[Tuple[torch.Tensor, torch.Tensor]] = None,
                attention_mask: Optional[torch.Tensor] = None, past_key_value: Any = None,
                cache_position: Optional[torch.Tensor] = None, **kw: Any) -> Tuple[torch.Tensor, dict]:
        x = hidden_states
        B, S, _ = x.shape
        H, KVH, Dh, C = self.nhead, self.kv_heads, self.head_dim, self.chunk_size
        start_pos = 0
        if cache_position is not None and cache_position.numel() > 0:
            start_pos = int(cache_position.reshape(-1)[0].item())
        router = self._get_router(past_key_value, B, x.dtype, x.device)
        if self.layer_idx == 0 and start_pos == 0:
            router.reset()
        cos, sin, rot_row0 = self._rotary_for(position_embeddings, start_pos, S, x.device)
        w, b = self._fused_qkv()
        qkv = F.linear(x, w, b)
        hp = self._cfg.hga_params(self._policy, B, x.dtype)
        qn = self.q_norm.weight if isinstance(self.q_norm, RMSNorm) else None
        kn = self.k_norm.weight if isinstance(self.k_norm, RMSNorm) else None
        qn = None if qn is None else qn.detach().to(x.dtype).contiguous()
        kn = None if kn is None else kn.detach().to(x.dtype).contiguous()
        out_heads = routed_attention(router, self.layer_idx, hp, qkv, cos, sin, rot_row0, start_pos, qn, kn,
                                     self.norm_eps, norm_mode=0, rope_mode=0, round_table=True)
        out = self.o_proj(out_heads.view(B, S, H * Dh))
        return out, {}
