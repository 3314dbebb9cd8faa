"""ctypes binding of libhga_b200.so (the C ABI declared in include/hga_b200.h).

The library is built in-tree by ``hierarchicalglobalattention_b200/build.py``.  There is no
fallback: if the shared object is missing or cannot be loaded, every op raises.
"""
from __future__ import annotations

import ctypes
import math
import os
import threading
from typing import Optional

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libhga_b200.so")

DTYPE_CODE = {torch.float32: 0, torch.bfloat16: 1, torch.float16: 2}

_lib = None
_lock = threading.Lock()


class HgaParams(ctypes.Structure):
    _fields_ = [
        ("batch", ctypes.c_int32), ("nhead", ctypes.c_int32), ("kv_heads", ctypes.c_int32),
        ("head_dim", ctypes.c_int32), ("chunk_size", ctypes.c_int32), ("group_size", ctypes.c_int32),
        ("topk_chunks", ctypes.c_int32), ("topk_groups", ctypes.c_int32), ("keep_first", ctypes.c_int32),
        ("keep_last", ctypes.c_int32), ("cutoff_pair", ctypes.c_int32), ("dtype", ctypes.c_int32),
        ("scale", ctypes.c_float), ("group_kv_scale", ctypes.c_float),
    ]


class HgaError(RuntimeError):
    """A libhga_b200 entry point returned an error code."""


_P, _I32, _I64, _F32P = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_void_p

_SIGNATURES = {
    "hga_version": (ctypes.c_char_p, []),
    "hga_last_error": (ctypes.c_char_p, []),
    "hga_summaries": (ctypes.c_int, [ctypes.POINTER(HgaParams), _I64, _I64, _P, _P, _P, _I64, _P, _P, _I32, _I64,
                                     _P, _P, _P, _I64, _I64, _P]),
    "hga_summaries_dual": (ctypes.c_int, [ctypes.POINTER(HgaParams), _I64, _I64, _P, _P, _P, _I64, _P, _P, _I64,
                                          _I32, _P, _P, _I64, _I64, _P, _P, _I64, _I64, _P, _P, _P, _I64, _I64,
                                          _P]),
    "hga_gather_h2d": (ctypes.c_int, [ctypes.POINTER(HgaParams), _P, _I32, _P, _P, _I64, _P, _P, _I32, _P, _P, _I64,
                                      _P, _I32, _P, _P, _P]),
    "hga_debug_fault": (ctypes.c_int, [_I32, _I64]),
    "hga_route_prefill": (ctypes.c_int, [ctypes.POINTER(HgaParams), _I64, _P, _I32, _P, _P, _I64, _P, _P, _P, _P,
                                         _P, _P, _P]),
    "hga_route_prefill_impl": (ctypes.c_int, [ctypes.POINTER(HgaParams), _I64, _P, _I32, _P, _P, _I64, _P, _P, _P,
                                              _P, _P, _P, _I32, _P]),
    "hga_attend_prefill": (ctypes.c_int, [ctypes.POINTER(HgaParams), _I64, _P, _I32, _P, _P, _I64, _P, _P, _P, _I32,
                                          _I32, _P]),
    "hga_route_decode": (ctypes.c_int, [ctypes.POINTER(HgaParams), _I32, _P, _P, _P, _P, _I64, _I32, _P, _P, _P, _P,
                                        _P]),
    "hga_attend_decode": (ctypes.c_int, [ctypes.POINTER(HgaParams), _I32, _P, _P, _P, _P, _I64, _I32, _P, _P, _I64,
                                         _P, _P, _I32, _P, _P]),
    "hga_attend_decode_dca": (ctypes.c_int, [ctypes.POINTER(HgaParams), _I32, _P, _P, _P, _P, _I64, _I32, _P, _P,
                                             _I64, _P, _P, _P, _I32, _P, _P, _I32, _I32, _P, _P]),
    "hga_route_prefill_range": (ctypes.c_int, [ctypes.POINTER(HgaParams), _I64, _I64, _I64, _P, _I32, _P, _P, _I64,
                                               _P, _P, _P, _P, _P, _P, _I32, _P]),
    "hga_attend_prefill_range": (ctypes.c_int, [ctypes.POINTER(HgaParams), _I64, _I64, _I64, _P, _I32, _P, _P, _I64,
                                                _P, _P, _P, _I32, _I32, _P]),
    "hga_shard_unpack": (ctypes.c_int, [_P, _I64, _I64, _I32, _I32, _P, _I64, _I64, _I64, _P, _P]),
    "hga_route_decode_impl": (ctypes.c_int, [ctypes.POINTER(HgaParams), _I32, _P, _P, _P, _P, _I64, _I32, _P, _P, _P,
                                             _P, _I32, _P]),
    "hga_attend_decode_impl": (ctypes.c_int, [ctypes.POINTER(HgaParams), _I32, _P, _P, _P, _P, _I64, _I32, _P, _P,
                                              _I64, _P, _P, _I32, _P, _I32, _P]),
    "hga_append_tokens": (ctypes.c_int, [ctypes.POINTER(HgaParams), _I32, _P, _P, _P, _P, _P, _P, _I64, _I32, _P, _P,
                                         _I64, _P, _P]),
    "hga_device_status": (ctypes.c_int, [_P, _I32]),
    "hga_qkv_prologue": (ctypes.c_int, [ctypes.POINTER(HgaParams), _I64, _P, _I64, _P, _P, ctypes.c_float, _I32, _P,
                                        _P, _I32, _I64, _I64, _P, _P, _P, _P, _I64, _I64, _P]),
}

ROT_F32, ROT_MODEL, ROT_F32_ROUNDED = 0, 1, 2


def exported_symbols():
    """Names of every entry point this binding expects the library to export."""
    return list(_SIGNATURES)


def lib():
    """Load (once) and return the ctypes handle; raises if the library is absent."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise HgaError(f"{LIB_PATH} is missing: run `python -m hierarchicalglobalattention_b200.build` "
                               "(the CUDA library is required; there is no CPU fallback)")
            h = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in _SIGNATURES.items():
                fn = getattr(h, name)
                fn.restype = res
                fn.argtypes = args
            _lib = h
    return _lib


def check(rc: int, what: str) -> None:
    if rc != 0:
        msg = lib().hga_last_error().decode(errors="replace")
        raise HgaError(f"{what} failed ({rc}): {msg}")


def stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def mixed_cutoff_pair(head_dim: int, chunk_size: int, theta: float, threshold: float = 0.5,
                      override: Optional[int] = None) -> int:
    """Number of RoPE pairs summed token-wise in a summary (vectorized.py:146-155)."""
    if override is not None:
        return int(override)
    half = head_dim // 2
    cutoff = 0
    for i in range(half):
        inv_freq = 1.0 / (theta ** (i / half))
        if max(1, chunk_size - 1) * inv_freq > threshold:
            cutoff = i + 1
    return cutoff


def make_params(*, batch, nhead, kv_heads, head_dim, chunk_size, group_size, topk_chunks, topk_groups,
                keep_first, keep_last, theta, dtype, mixed_rope_threshold=0.5, mixed_rope_cutoff_pair=None):
    return HgaParams(
        batch=batch, nhead=nhead, kv_heads=kv_heads, head_dim=head_dim, chunk_size=chunk_size,
        group_size=group_size, topk_chunks=topk_chunks, topk_groups=topk_groups,
        keep_first=max(0, int(keep_first)), keep_last=max(0, int(keep_last)),
        cutoff_pair=mixed_cutoff_pair(head_dim, chunk_size, theta, mixed_rope_threshold, mixed_rope_cutoff_pair),
        dtype=DTYPE_CODE[dtype], scale=head_dim ** -0.5,
        group_kv_scale=1.0 / (group_size + math.sqrt(group_size)),
    )


def device_status(clear: bool = True) -> int:
    """First device error code of the kernels (0 = none): a bounded tensor-core wait that timed out,
    or a decode bounds check (0x101 routing, 0x102 attention, 0x103 append)."""
    code = ctypes.c_int32(0)
    check(lib().hga_device_status(ctypes.byref(code), 1 if clear else 0), "hga_device_status")
    return int(code.value)
