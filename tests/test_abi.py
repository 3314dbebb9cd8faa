"""The C-ABI library loads and exports every entry point include/hga_b200.h declares (no GPU)."""
import ctypes
import os
import re

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared():
    names = []
    for fn in sorted(os.listdir(os.path.join(ROOT, "include"))):
        if fn.endswith(".h"):
            src = open(os.path.join(ROOT, "include", fn)).read()
            src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
            names += re.findall(r"\b(hga_[a-z0-9_]+)\s*\(", src)
    return sorted(set(names))


def test_library_exports_every_declared_symbol():
    from hierarchicalglobalattention_b200 import _lib
    h = _lib.lib()
    declared = _declared()
    assert declared, "no declarations found"
    missing = [n for n in declared if not hasattr(h, n)]
    assert not missing, missing
    assert set(_lib.exported_symbols()) <= set(declared)


def test_invalid_arguments_fail_loudly_without_touching_the_device():
    from hierarchicalglobalattention_b200 import _lib
    h = _lib.lib()
    rc = h.hga_summaries(None, 10, 0, None, None, None, 10, None, None, 0, 0, None, None, None, 1, 0, None)
    assert rc == -1 and b"NULL" in h.hga_last_error()
    p = _lib.make_params(batch=1, nhead=3, kv_heads=2, head_dim=16, chunk_size=8, group_size=4, topk_chunks=1,
                         topk_groups=2, keep_first=0, keep_last=0, theta=1e4, dtype=__import__("torch").float32)
    rc = h.hga_route_prefill(ctypes.byref(p), 16, 1, 0, 1, 1, 2, 1, 1, 1, 1, None, None, None)
    assert rc == -1 and b"kv_heads" in h.hga_last_error()


def test_ops_refuse_cpu_tensors():
    import torch
    from hierarchicalglobalattention_b200 import _lib, ops
    p = _lib.make_params(batch=1, nhead=2, kv_heads=1, head_dim=16, chunk_size=8, group_size=4, topk_chunks=1,
                         topk_groups=2, keep_first=0, keep_last=0, theta=1e4, dtype=torch.float32)
    k = torch.zeros(1, 1, 16, 16)
    with pytest.raises(_lib.HgaError, match="CUDA"):
        ops.summaries(p, k, k, k, torch.zeros(16, 16), torch.zeros(16, 16))


def test_module_state_dict_loads_from_reference_layout():
    import hierarchicalglobalattention_b200 as hga
    m = hga.HierarchicalGlobalAttentionRouted(d_model=256, nhead=4, kv_heads=2, qk_norm=True)
    names = set(m.state_dict())
    assert names == {"q_proj.weight", "k_proj.weight", "v_proj.weight", "o_proj.weight", "q_norm.weight",
                     "k_norm.weight"}


def test_module_fails_loudly_on_cpu():
    import hierarchicalglobalattention_b200 as hga
    m = hga.HierarchicalGlobalAttentionRouted(d_model=64, nhead=4, kv_heads=2)
    with pytest.raises(Exception, match="CUDA"):
        m(torch.randn(1, 130, 64))


def test_qwen_patch_host_side():
    """rope theta from both HF config styles; replace/restore bookkeeping (no kernels run)."""
    import types
    import torch.nn as nn
    from hierarchicalglobalattention_b200.qwen import (QwenRoutedAttention, replace_qwen_attention_with_router,
                                                       restore_original_attention, rope_theta_of)
    assert rope_theta_of(types.SimpleNamespace(rope_parameters={"rope_theta": 5e5})) == 5e5
    assert rope_theta_of(types.SimpleNamespace(rope_theta=1e4)) == 1e4
    assert rope_theta_of(types.SimpleNamespace()) == 1e6
    cfg = types.SimpleNamespace(num_attention_heads=4, num_key_value_heads=2, head_dim=16, hidden_size=64,
                                num_hidden_layers=2, rope_parameters={"rope_theta": 1e4})

    class Attn(nn.Module):
        def __init__(self, i):
            super().__init__()
            self.layer_idx = i
            self.q_proj, self.k_proj = nn.Linear(64, 64, bias=False), nn.Linear(64, 32, bias=False)
            self.v_proj, self.o_proj = nn.Linear(64, 32, bias=False), nn.Linear(64, 64, bias=False)

    model = nn.Module()
    model.config = cfg
    model.model = nn.Module()
    model.model.layers = nn.ModuleList()
    for i in range(2):
        layer = nn.Module()
        layer.self_attn = Attn(i)
        model.model.layers.append(layer)
    n_params = sum(p.numel() for p in model.parameters())
    assert replace_qwen_attention_with_router(model, topk_chunks=3) == 2
    assert replace_qwen_attention_with_router(model, topk_chunks=3) == 2          # idempotent
    w = model.model.layers[1].self_attn
    assert isinstance(w, QwenRoutedAttention) and w.layer_idx == 1 and w._cfg.theta == 1e4
    assert sum(p.numel() for p in model.parameters()) == n_params                 # no new parameters
    assert restore_original_attention(model) == 2
    assert isinstance(model.model.layers[0].self_attn, Attn)


def _p(**kw):
    from hierarchicalglobalattention_b200 import _lib
    base = dict(batch=1, nhead=4, kv_heads=2, head_dim=16, chunk_size=8, group_size=4, topk_chunks=2,
                topk_groups=4, keep_first=1, keep_last=1, theta=1e4, dtype=torch.float32)
    base.update(kw)
    return _lib.make_params(**base)


def test_range_decode_and_unpack_entry_points_validate_before_any_launch():
    """Bad ranges, impl choices, positions lists and unpack layouts are rejected with a message
    naming the problem; none of these calls reaches the device."""
    from hierarchicalglobalattention_b200 import _lib
    h = _lib.lib()
    p = _p()
    P = ctypes.byref(p)
    one = ctypes.c_void_p(16)  # any non-NULL pointer: validation fails before it is used
    # query-chunk range outside the sequence / empty
    rc = h.hga_route_prefill_range(P, 40, 3, 9, one, 0, one, one, 8, one, one, one, one, None, None, 0, None)
    assert rc == -1 and b"range" in h.hga_last_error()
    rc = h.hga_attend_prefill_range(P, 40, 2, 2, one, 0, one, one, 64, one, one, one, 1, 0, None)
    assert rc == -1 and b"range" in h.hga_last_error()
    # unknown kernel choice
    rc = h.hga_route_decode_impl(P, 1, one, one, one, one, 8, 4, one, one, one, one, 7, None)
    assert rc == -1 and b"impl" in h.hga_last_error()
    rc = h.hga_attend_decode_impl(P, 1, one, one, one, one, 64, 0, one, one, 64, one, one, 4, one, 9, None)
    assert rc == -1 and b"impl" in h.hga_last_error()
    # a fast kernel asked for where it does not apply (fp32, head_dim 16)
    rc = h.hga_attend_decode_impl(P, 1, one, one, one, one, 64, 0, one, one, 64, one, one, 4, one, 2, None)
    assert rc == -2 and b"fast kernel" in h.hga_last_error()
    # decode block longer than a chunk, unknown hot_mode
    rc = h.hga_append_tokens(P, 9, one, one, one, None, one, one, 64, 0, None, None, 0, None, None)
    assert rc == -1 and b"chunk_size" in h.hga_last_error()
    rc = h.hga_append_tokens(P, 1, one, one, one, None, one, one, 64, 3, None, None, 0, None, None)
    assert rc == -1 and b"hot_mode" in h.hga_last_error()
    # unpack: misaligned row size, out-of-range destination block
    tab = (ctypes.c_int32 * 4)(0, 3, 1, 2)
    rc = h.hga_shard_unpack(one, 64, 0, 2, 2, ctypes.cast(tab, ctypes.c_void_p), 1, 4, 24, one, None)
    assert rc == -1 and b"aligned" in h.hga_last_error()
    bad = (ctypes.c_int32 * 4)(0, 3, 1, 7)
    rc = h.hga_shard_unpack(one, 64, 0, 2, 2, ctypes.cast(bad, ctypes.c_void_p), 1, 4, 32, one, None)
    assert rc == -1 and b"block" in h.hga_last_error()


def test_host_size_rules_match_the_reference():
    """(N, Kc, Kg, Kg_request) of a prefill and (Kc, Kg) of a decode block: vectorized.py:304,
    365-366 and chunk_router.py:226, 256."""
    from hierarchicalglobalattention_b200 import ops
    p = _p(chunk_size=64, group_size=16, topk_chunks=16, topk_groups=64)
    assert ops.route_sizes(p, 32768) == (512, 16, 64, 32)
    assert ops.route_sizes(p, 100) == (2, 2, 8, 8)
    assert ops.route_sizes(_p(chunk_size=64, group_size=16, topk_chunks=16, topk_groups=1), 4096)[2] == 0
    assert ops.decode_sizes(p, 502) == (16, 64)
    assert ops.decode_sizes(p, 3) == (3, 12)
    assert ops.decode_sizes(_p(topk_chunks=0), 10) == (0, 0)
