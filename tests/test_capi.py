"""CPU checks of the C-ABI library: it loads, exports every symbol that
include/poly_attention.h declares, agrees on struct layouts, and the product
path refuses CPU tensors (there is no CPU implementation)."""
import ctypes
import os
import re

import pytest
import torch

from conftest import ROOT

HEADER = os.path.join(ROOT, "include", "poly_attention.h")


def declared():
    src = open(HEADER).read()
    return re.findall(r"POLY_API\s+[\w\s\*]+?\b(poly_\w+)\s*\(", src)


def test_header_declares_entry_points():
    names = declared()
    assert {"poly_pass_fwd", "poly_pass_bwd", "poly_lse_merge", "poly_last_error"} <= set(names)


def test_library_exports_every_declared_symbol():
    from poly_attention_b200 import _lib
    for name in declared():
        assert hasattr(_lib.lib, name), name
        assert name in _lib.EXPORTS, f"{name} is not bound in _lib.EXPORTS"


def test_struct_layout_matches():
    from poly_attention_b200 import _lib
    assert _lib.lib.poly_sizeof_pass_args() == ctypes.sizeof(_lib.PolyPassArgs)
    assert _lib.lib.poly_sizeof_pass_bwd_args() == ctypes.sizeof(_lib.PolyPassBwdArgs)
    assert _lib.lib.poly_sizeof_merge_args() == ctypes.sizeof(_lib.PolyMergeArgs)
    assert _lib.lib.poly_abi_version() == _lib.ABI_VERSION


def test_invalid_args_report_errors_without_gpu():
    from poly_attention_b200 import _lib
    a = _lib.PolyPassArgs()
    rc = _lib.lib.poly_pass_fwd(ctypes.byref(a), None)
    assert rc == _lib.POLY_EINVAL
    assert "positive" in _lib.lib.poly_last_error().decode()
    a.batch = a.heads = a.kv_heads = a.seq_q = a.seq_k = 1
    a.head_dim, a.heads, a.kv_heads = 64, 3, 2
    assert _lib.lib.poly_pass_fwd(ctypes.byref(a), None) == _lib.POLY_EINVAL
    assert "divisible" in _lib.lib.poly_last_error().decode()
    a.heads, a.head_dim = 2, 512
    assert _lib.lib.poly_pass_fwd(ctypes.byref(a), None) == _lib.POLY_EUNSUPPORTED
    # causal_offset: negative is invalid; non-zero is refused (before any launch)
    # outside the tcgen05 forward, here an fp32 pass
    a.head_dim, a.q, a.k, a.v, a.out = 64, 256, 256, 256, 256
    a.causal, a.causal_offset = 1, -128
    assert _lib.lib.poly_pass_fwd(ctypes.byref(a), None) == _lib.POLY_EINVAL
    assert "causal_offset" in _lib.lib.poly_last_error().decode()
    a.dtype, a.causal_offset = _lib.POLY_F32, 128
    assert _lib.lib.poly_pass_fwd(ctypes.byref(a), None) == _lib.POLY_EUNSUPPORTED
    assert "causal_offset" in _lib.lib.poly_last_error().decode()
    a.causal_offset, a.q, a.k, a.v, a.out, a.head_dim = 0, None, None, None, None, 512
    # poly_copy_rows validates every copy before launching
    rc = _lib.PolyRowCopy()
    assert _lib.lib.poly_copy_rows(None, 1, None) == _lib.POLY_EINVAL
    assert _lib.lib.poly_copy_rows(ctypes.byref(rc), 17, None) == _lib.POLY_EINVAL
    assert _lib.lib.poly_copy_rows(ctypes.byref(rc), 0, None) == _lib.POLY_OK
    rc.outer, rc.inner, rc.row_bytes, rc.src, rc.dst = 2, 2, 24, 16, 32
    assert _lib.lib.poly_copy_rows(ctypes.byref(rc), 1, None) == _lib.POLY_EINVAL
    assert "16-byte" in _lib.lib.poly_last_error().decode()
    # poly_decode_chain validates every pass before launching any
    assert _lib.lib.poly_decode_chain(None, 1, None) == _lib.POLY_EINVAL
    assert _lib.lib.poly_decode_chain(ctypes.byref(a), -1, None) == _lib.POLY_EINVAL
    assert _lib.lib.poly_decode_chain(ctypes.byref(a), 0, None) == _lib.POLY_OK
    assert _lib.lib.poly_decode_chain(ctypes.byref(a), 1, None) == _lib.POLY_EUNSUPPORTED


def test_product_path_refuses_cpu_tensors():
    import poly_attention_b200 as P
    q = torch.randn(1, 2, 8, 32)
    with pytest.raises(RuntimeError, match="CUDA"):
        P.flash_poly_attention(q, q, q, q)
    with pytest.raises(RuntimeError, match="CUDA"):
        P.PolyAttention(dim=64, heads=2, dim_head=32)(torch.randn(1, 8, 64))


def test_flash_rejects_context_mask_like_reference():
    # poly_attention/flash_poly_attention.py:455 ; tests/test_poly_attention.py:541-552
    import poly_attention_b200 as P
    q = torch.randn(2, 4, 16, 32)
    cm = (torch.ones(2, 16, dtype=torch.bool), torch.ones(2, 16, dtype=torch.bool))
    with pytest.raises(AssertionError, match="context_mask is not supported"):
        P.flash_poly_attention(q, q, q, q, context_mask=cm)


def test_module_error_contracts():
    # tests/test_poly_attention.py:578-586 and the constructor asserts
    import poly_attention_b200 as P
    attn = P.PolyAttention(dim=64, heads=4, multiply_root_value=True)
    x = torch.randn(2, 16, 64)
    with pytest.raises(AssertionError, match="first context sequence length"):
        attn(x, context=(torch.randn(2, 20, 64), torch.randn(2, 24, 64)))
    with pytest.raises(AssertionError, match="divisible"):
        P.PolyAttention(dim=64, heads=4, kv_heads=3)
    with pytest.raises(AssertionError, match="root value"):
        P.NPolyAttention(dim=64, heads=4, kv_heads=2, use_root_value_as_attn_gate=True)


def test_state_dict_names_match_reference(golden):
    import poly_attention_b200 as P
    g = golden("mod2_causal_gqa")
    ref_keys = {k[2:] for k in g if k.startswith("p:")}
    m = P.PolyAttention(dim=64, heads=4, kv_heads=2, dim_head=16, causal=True, softclamp_value=20.0)
    assert set(m.state_dict()) == ref_keys
    g = golden("modn_o3_g2")
    ref_keys = {k[2:] for k in g if k.startswith("p:")}
    m = P.NPolyAttention(dim=64, order=3, heads=4, kv_heads=2, dim_head=16, causal=True)
    assert set(m.state_dict()) == ref_keys


def test_polyvit_state_dict_names_match_reference(golden):
    import poly_attention_b200 as P
    for order in (2, 3):
        g = golden(f"vit_o{order}")
        ref_keys = {k[2:] for k in g if k.startswith("p:")}
        m = P.PolyViT(image_size=32, patch_size=8, num_classes=10, dim=64, depth=2, heads=4, mlp_dim=128,
                      dim_head=16, order=order)
        assert set(m.state_dict()) == ref_keys
