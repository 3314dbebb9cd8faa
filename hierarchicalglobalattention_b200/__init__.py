"""B200-native (sm_100a) implementation of HGA's routed-attention hot path.

Drop-in for the reference's ``HierarchicalGlobalAttentionRouted`` module, its ``KvRouter``
(``ChunkRouter`` / ``RoutedKV`` / ``RouterConfig`` / KV-cache stores) and its Qwen3 patch
(``replace_qwen_attention_with_router``).  Compute runs in hand-written CUDA kernels behind the C
ABI of ``libhga_b200.so`` (include/hga_b200.h); PyTorch provides device memory, streams and the
projection GEMMs.
"""
from . import _lib, ops, torch_ops  # noqa: F401  (torch_ops registers torch.ops.hga.*)
from .config import ChunkPlacementPolicy, RouterConfig
from .module import HierarchicalGlobalAttentionRouted
from .router import ChunkRouter, RoutedKV
from .qwen import QwenRoutedAttention, replace_qwen_attention_with_router, restore_original_attention
from .store import KVCacheStore, VramKVCacheStore
from .store_ram import RamKVCacheStore

__all__ = ["ChunkPlacementPolicy", "RouterConfig", "HierarchicalGlobalAttentionRouted", "ChunkRouter",
           "RoutedKV", "KVCacheStore", "VramKVCacheStore", "RamKVCacheStore", "QwenRoutedAttention",
           "replace_qwen_attention_with_router", "restore_original_attention", "ops"]
