"""ctypes binding of libpolyattn.so (declarations: include/poly_attention.h).

The library is the only implementation: if it is missing, importing this
module raises, there is no fallback.
"""
from __future__ import annotations

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libpolyattn.so")

POLY_OK, POLY_EINVAL, POLY_EUNSUPPORTED, POLY_ECUDA = 0, 1, 2, 3
POLY_F32, POLY_F16, POLY_BF16 = 0, 1, 2
ABI_VERSION = 2

c_i32, c_i64, c_f32, c_vp, c_sz = ctypes.c_int32, ctypes.c_int64, ctypes.c_float, ctypes.c_void_p, ctypes.c_size_t
I64x3 = c_i64 * 3
I64x2 = c_i64 * 2


class PolyPassArgs(ctypes.Structure):
    _fields_ = [
        ("batch", c_i32), ("heads", c_i32), ("kv_heads", c_i32), ("seq_q", c_i32), ("seq_k", c_i32),
        ("head_dim", c_i32), ("dtype", c_i32), ("causal", c_i32), ("scale", c_f32), ("softclamp", c_f32),
        ("q", c_vp), ("q_stride", I64x3),
        ("k", c_vp), ("k_stride", I64x3),
        ("v", c_vp), ("v_stride", I64x3),
        ("v_mul", c_vp), ("v_mul_stride", I64x3),
        ("bias", c_vp), ("bias_stride", I64x2),
        ("key_mask", c_vp), ("key_mask_stride", c_i64),
        ("query_mask", c_vp), ("query_mask_stride", c_i64),
        ("out", c_vp), ("out_stride", I64x3),
        ("lse", c_vp), ("lse_stride", I64x2),
        ("epi_mul", c_vp), ("epi_mul_stride", I64x3),
        ("epi_out", c_vp), ("epi_out_stride", I64x3),
        ("workspace", c_vp), ("workspace_bytes", c_sz),
        ("causal_offset", c_i32), ("reserved_", c_i32),
    ]


class PolyPassBwdArgs(ctypes.Structure):
    _fields_ = [
        ("fwd", PolyPassArgs),
        ("dout", c_vp), ("dout_stride", I64x3),
        ("dlse", c_vp), ("dlse_stride", I64x2),
        ("dq", c_vp), ("dq_stride", I64x3),
        ("dk", c_vp), ("dk_stride", I64x3),
        ("dv", c_vp), ("dv_stride", I64x3),
        ("dbias", c_vp), ("dbias_stride", I64x2),
        ("dq_accumulate", c_i32), ("reserved", c_i32),
        ("workspace", c_vp), ("workspace_bytes", c_sz),
    ]


class PolyMergeArgs(ctypes.Structure):
    _fields_ = [
        ("parts", c_i32), ("head_dim", c_i32), ("dtype", c_i32), ("reserved", c_i32), ("rows", c_i64),
        ("part_out", c_vp), ("part_lse", c_vp), ("out", c_vp), ("lse", c_vp),
    ]


class PolyRowCopy(ctypes.Structure):
    _fields_ = [("src", c_vp), ("dst", c_vp), ("outer", ctypes.c_int32), ("inner", ctypes.c_int32),
                ("row_bytes", ctypes.c_int32), ("reserved", ctypes.c_int32),
                ("src_stride", ctypes.c_int64 * 2), ("dst_stride", ctypes.c_int64 * 2)]


MAX_ROW_COPIES = 16


class PolyHeadNorm(ctypes.Structure):
    _fields_ = [("src", c_vp), ("dst", c_vp), ("weight", c_vp), ("batch", ctypes.c_int32),
                ("heads", ctypes.c_int32), ("rows", ctypes.c_int32), ("dim", ctypes.c_int32),
                ("src_stride", ctypes.c_int64 * 3), ("src_dtype", ctypes.c_int32), ("dst_dtype", ctypes.c_int32),
                ("weight_dtype", ctypes.c_int32), ("eps", ctypes.c_float)]


MAX_NORMS = 4

EXPORTS = {
    "poly_pass_fwd": (ctypes.c_int, [ctypes.POINTER(PolyPassArgs), c_vp]),
    "poly_pass_fwd_workspace_size": (c_sz, [ctypes.POINTER(PolyPassArgs)]),
    "poly_pass_bwd": (ctypes.c_int, [ctypes.POINTER(PolyPassBwdArgs), c_vp]),
    "poly_pass_bwd_workspace_size": (c_sz, [ctypes.POINTER(PolyPassBwdArgs)]),
    "poly_lse_merge": (ctypes.c_int, [ctypes.POINTER(PolyMergeArgs), c_vp]),
    "poly_decode_chain": (ctypes.c_int, [ctypes.POINTER(PolyPassArgs), ctypes.c_int, c_vp]),
    "poly_copy_rows": (ctypes.c_int, [ctypes.POINTER(PolyRowCopy), ctypes.c_int, c_vp]),
    "poly_head_rmsnorm": (ctypes.c_int, [ctypes.POINTER(PolyHeadNorm), ctypes.c_int, c_vp]),
    "poly_pass_bwd_noalloc": (ctypes.c_int, [ctypes.POINTER(PolyPassBwdArgs), c_vp]),
    "poly_noalloc_scratch_bytes": (c_sz, []),
    "poly_pass_fwd_kernel_name": (ctypes.c_char_p, [ctypes.POINTER(PolyPassArgs)]),
    "poly_pass_bwd_kernel_name": (ctypes.c_char_p, [ctypes.POINTER(PolyPassBwdArgs)]),
    "poly_last_error": (ctypes.c_char_p, []),
    "poly_launch_count": (ctypes.c_ulonglong, []),
    "poly_device_error": (ctypes.c_int, [ctypes.POINTER(ctypes.c_int), ctypes.c_int]),
    "poly_selftest_wait_timeout": (ctypes.c_int, [ctypes.c_ulonglong, c_vp, c_vp]),
    "poly_abi_version": (ctypes.c_int, []),
    "poly_sizeof_pass_args": (c_sz, []),
    "poly_sizeof_pass_bwd_args": (c_sz, []),
    "poly_sizeof_merge_args": (c_sz, []),
}


def _load():
    if not os.path.exists(LIB_PATH):
        raise ImportError(f"{LIB_PATH} is missing: build it with `python poly-attention_b200/build.py` "
                          "(there is no non-CUDA implementation)")
    lib = ctypes.CDLL(LIB_PATH)
    for name, (res, args) in EXPORTS.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    if lib.poly_abi_version() != ABI_VERSION:
        raise ImportError("libpolyattn.so ABI version mismatch")
    for fn, st in (("poly_sizeof_pass_args", PolyPassArgs), ("poly_sizeof_pass_bwd_args", PolyPassBwdArgs),
                   ("poly_sizeof_merge_args", PolyMergeArgs)):
        if getattr(lib, fn)() != ctypes.sizeof(st):
            raise ImportError(f"libpolyattn.so struct layout mismatch ({st.__name__})")
    return lib


lib = _load()


def check(rc: int, what: str):
    if rc == POLY_OK:
        return
    msg = f"{what}: {lib.poly_last_error().decode()}"
    if rc == POLY_EINVAL:
        raise ValueError(msg)
    if rc == POLY_EUNSUPPORTED:
        raise NotImplementedError(msg)
    raise RuntimeError(msg)


def launch_count() -> int:
    """Kernels launched by libpolyattn.so in this process so far."""
    return int(lib.poly_launch_count())


def device_error(reset: bool = False) -> int:
    """Device error word (non-zero: a bounded in-kernel wait gave up)."""
    v = ctypes.c_int(0)
    check(lib.poly_device_error(ctypes.byref(v), int(reset)), "poly_device_error")
    return v.value
