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

Not carried over (outside the token-only routed hot path): the Dual Chunk Attention variant
(``dca_chunk > 0``) and the file-system cache tier (``cache_location="fs"``); both raise.
"""
from __future__ import annotations

from typing import Any, Optional, Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F

from .config import ChunkPlacementPolicy, RouterConfig
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


class QwenRoutedAttention(nn.Module):
    """Replacement for ``Qwen3MoeAttention`` / ``Qwen3Attention`` routing through a shared
    ``ChunkRouter``; adds no parameters."""

    def __init__(self, orig: nn.Module, config: Any, *, chunk_size: int = 64, group_size: int = 16,
                 keep_first: int = 2, keep_last: int = 2, topk_chunks: int = 8, topk_groups: int = 32,
                 cache_location: str = "vram", vram_cache_chunks: int = 256, vram_summary_chunks: int = 4096,
                 vram_cache_reserve_gb: float = 1.5, ram_budget_gb: float = 12.0,
                 fs_cache_dir: Optional[str] = None, dca_chunk: int = 0, dca_local: int = 0) -> None:
        super().__init__()
        if dca_chunk > 0:
            raise NotImplementedError("Dual Chunk Attention (dca_chunk > 0) is not part of the B200 routed path")
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
        self.dca_chunk, self.dca_local = 0, 0
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
