"""Incremental (single active chunk) routing + attention.  Device kernels land here."""
from __future__ import annotations


def decode_block(router, layer, q, k_rope, k_raw, v, start_pos):
    raise NotImplementedError("incremental decode path is not built yet")
