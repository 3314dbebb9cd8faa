"""Host-side checks of the Dual Chunk Attention path (no kernels run): argument validation of the
wrapper and of the C entry point, and the fp32 RoPE table against the wrapper's formula."""
import types

import pytest
import torch

from oracle import hga_oracle as O


def test_wrapper_rejects_dca_chunk_not_multiple_of_chunk_size():
    from hierarchicalglobalattention_b200.qwen import QwenRoutedAttention
    cfg = types.SimpleNamespace(num_attention_heads=4, num_key_value_heads=2, head_dim=16, hidden_size=64,
                                num_hidden_layers=1, rope_theta=1e4)
    with pytest.raises(ValueError, match="multiple of chunk_size"):
        QwenRoutedAttention(torch.nn.Module(), cfg, chunk_size=64, dca_chunk=100)
    w = QwenRoutedAttention(torch.nn.Module(), cfg, chunk_size=16, dca_chunk=64)
    assert (w.dca_local, w.dca_ceil) == (12, 76)          # default local window: a fifth of the chunk
    w = QwenRoutedAttention(torch.nn.Module(), cfg, chunk_size=16, dca_chunk=64, dca_local=3)
    assert (w.dca_local, w.dca_ceil) == (3, 67)


def test_entry_point_rejects_bad_dca_arguments():
    from hierarchicalglobalattention_b200 import _lib, ops
    p = _lib.make_params(batch=1, nhead=4, kv_heads=2, head_dim=16, chunk_size=16, group_size=4, topk_chunks=2,
                         topk_groups=2, keep_first=1, keep_last=1, theta=1e4, dtype=torch.float32)
    lib = _lib.lib()
    args = lambda chunk, ceil, dh_p=p: (ops.ctypes_params(dh_p), 1, 16, 16, 16, 16, 16, 0, None, None, 16, None, None,
                                        None, 0, 16, 16, chunk, ceil, 16, None)
    assert lib.hga_attend_decode_dca(*args(0, 0)) != 0 and b"dca_chunk" in lib.hga_last_error()
    assert lib.hga_attend_decode_dca(*args(64, 32)) != 0 and b"dca_ceil" in lib.hga_last_error()


def test_rope_table_equals_the_wrapper_formula():
    from hierarchicalglobalattention_b200 import ops
    c, s = ops.dca_rope_table(76, 64, 1e6, torch.device("cpu"))
    pos = torch.tensor([0, 5, 63, 64, 76])
    rc, rs = O.dca_rope_table(pos, 64, 1e6, torch.float32)
    assert torch.equal(c[pos], rc) and torch.equal(s[pos], rs)
