"""Torch-facing wrappers around the C ABI (one attention pass, its backward,
the key-split merge). Tensors must live on a CUDA device; they are passed to
the library as raw pointers plus (batch, head, row) element strides, so the
projections' natural [b, n, h, d] memory layout is consumed without copies.
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib
from ._lib import PolyMergeArgs, PolyPassArgs, PolyPassBwdArgs, check, lib

_DTYPES = {torch.float32: _lib.POLY_F32, torch.float16: _lib.POLY_F16, torch.bfloat16: _lib.POLY_BF16}


def _require_cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise RuntimeError("poly_attention_b200 runs on CUDA tensors only (no CPU implementation)")


def _rows(t):
    """Make the last dim contiguous; return (tensor, stride3)."""
    if t.stride(-1) != 1:
        t = t.contiguous()
    return t, (t.stride(0), t.stride(1), t.stride(2))


def _vec(t):
    if t is None:
        return None, (0, 0)
    if t.dtype != torch.float32:
        t = t.float()
    if t.stride(-1) != 1:
        t = t.contiguous()
    return t, (t.stride(0), t.stride(1))


def _mask(m, n):
    if m is None:
        return None, 0
    m = m.to(torch.uint8)
    if m.stride(-1) != 1:
        m = m.contiguous()
    if m.shape[-1] != n:
        raise ValueError(f"mask length {m.shape[-1]} does not match sequence length {n}")
    return m, m.stride(0)


def _stream(device):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _ptr(t):
    return None if t is None else t.data_ptr()


def _fill_pass(a: PolyPassArgs, q, k, v, out, lse, *, causal, softclamp, scale, bias, key_mask, query_mask,
               epi_mul, epi_out, keep, v_mul=None):
    b, h, nq, d = q.shape
    _, g, nk, _ = k.shape
    a.batch, a.heads, a.kv_heads, a.seq_q, a.seq_k, a.head_dim = b, h, g, nq, nk, d
    a.dtype = _DTYPES[q.dtype]
    a.causal = int(bool(causal))
    a.scale = float(d ** -0.5 if scale is None else scale)
    a.softclamp = float(softclamp) if softclamp else 0.0
    q, a.q_stride = _rows(q)
    k, a.k_stride = _rows(k)
    v, a.v_stride = _rows(v)
    a.q, a.k, a.v = _ptr(q), _ptr(k), _ptr(v)
    if v_mul is not None:
        v_mul, a.v_mul_stride = _rows(v_mul)
        a.v_mul = _ptr(v_mul)
    bias, a.bias_stride = _vec(bias)
    a.bias = _ptr(bias)
    key_mask, a.key_mask_stride = _mask(key_mask, nk)
    query_mask, a.query_mask_stride = _mask(query_mask, nq)
    a.key_mask, a.query_mask = _ptr(key_mask), _ptr(query_mask)
    a.out, a.out_stride = _ptr(out), (out.stride(0), out.stride(1), out.stride(2))
    if lse is not None:
        a.lse, a.lse_stride = _ptr(lse), (lse.stride(0), lse.stride(1))
    if epi_out is not None:
        epi_mul, a.epi_mul_stride = _rows(epi_mul)
        a.epi_mul, a.epi_out = _ptr(epi_mul), _ptr(epi_out)
        a.epi_out_stride = (epi_out.stride(0), epi_out.stride(1), epi_out.stride(2))
    keep.extend([q, k, v, bias, key_mask, query_mask, epi_mul, v_mul])


@torch.compiler.disable   # library calls through ctypes: dynamo runs them eagerly
def pass_fwd(q, k, v, *, causal=False, softclamp=None, scale=None, bias=None, key_mask=None, query_mask=None,
             epi_mul=None, v_mul=None, out=None, lse=None, want_lse=True, causal_offset=0):
    """One attention pass (see PolyPassArgs in include/poly_attention.h).

    ``causal_offset`` (with causal, a multiple of 128): key j is visible to
    query i iff j <= i + causal_offset.

    ``v_mul`` (same shape as v) multiplies the values elementwise inside the
    kernel; ``epi_mul`` (shape of out) makes the kernel also return epi_mul * out.

    q [b, h, nq, d]; k, v [b, g, nk, d] with g | h; bias [b, g, nk] fp32.
    Returns (out, lse[, epi_out]) with out in q's dtype and lse fp32 [b, h, nq].
    """
    _require_cuda(q, k, v, bias, key_mask, query_mask, epi_mul, v_mul)
    if q.dtype not in _DTYPES or k.dtype != q.dtype or v.dtype != q.dtype:
        raise TypeError(f"q, k, v must share one of {list(_DTYPES)}; got {q.dtype}, {k.dtype}, {v.dtype}")
    b, h, nq, d = q.shape
    if out is None:
        out = torch.empty(b, h, nq, d, device=q.device, dtype=q.dtype)
    if lse is None and want_lse:
        lse = torch.empty(b, h, nq, device=q.device, dtype=torch.float32)
    epi_out = torch.empty_like(out) if epi_mul is not None else None
    a = PolyPassArgs()
    keep = []
    _fill_pass(a, q, k, v, out, lse, causal=causal, softclamp=softclamp, scale=scale, bias=bias, key_mask=key_mask,
               query_mask=query_mask, epi_mul=epi_mul, epi_out=epi_out, keep=keep, v_mul=v_mul)
    a.causal_offset = int(causal_offset)
    ws_bytes = lib.poly_pass_fwd_workspace_size(ctypes.byref(a))
    ws = None
    if ws_bytes:
        ws = torch.empty(ws_bytes, device=q.device, dtype=torch.uint8)
        a.workspace, a.workspace_bytes = ws.data_ptr(), ws_bytes
    check(lib.poly_pass_fwd(ctypes.byref(a), _stream(q.device)), "poly_pass_fwd")
    if epi_mul is not None:
        return out, lse, epi_out
    return out, lse


@torch.compiler.disable
def pass_bwd(q, k, v, out, lse, dout, *, causal=False, softclamp=None, scale=None, bias=None, key_mask=None,
             query_mask=None, dlse=None, dq=None, dq_accumulate=False, want_dbias=False):
    """Backward of ``pass_fwd``. Returns (dq, dk, dv, dbias-or-None)."""
    _require_cuda(q, k, v, out, lse, dout, dlse)
    a = PolyPassBwdArgs()
    keep = []
    _fill_pass(a.fwd, q, k, v, out, lse, causal=causal, softclamp=softclamp, scale=scale, bias=bias,
               key_mask=key_mask, query_mask=query_mask, epi_mul=None, epi_out=None, keep=keep)
    if out.stride(-1) != 1 or lse.stride(-1) != 1:
        raise ValueError("out and lse must have a contiguous last dim")
    dout, a.dout_stride = _rows(dout.to(q.dtype))
    a.dout = _ptr(dout)
    dlse, a.dlse_stride = _vec(dlse)
    a.dlse = _ptr(dlse)
    if dq is None:
        dq = torch.empty_like(q)
    dk = torch.empty_like(k, memory_format=torch.contiguous_format)
    dv = torch.empty_like(v, memory_format=torch.contiguous_format)
    dbias = torch.empty(k.shape[:3], device=q.device, dtype=torch.float32) if want_dbias else None
    a.dq, a.dq_stride = _ptr(dq), (dq.stride(0), dq.stride(1), dq.stride(2))
    a.dk, a.dk_stride = _ptr(dk), (dk.stride(0), dk.stride(1), dk.stride(2))
    a.dv, a.dv_stride = _ptr(dv), (dv.stride(0), dv.stride(1), dv.stride(2))
    if dbias is not None:
        a.dbias, a.dbias_stride = _ptr(dbias), (dbias.stride(0), dbias.stride(1))
    a.dq_accumulate = int(bool(dq_accumulate))
    ws_bytes = lib.poly_pass_bwd_workspace_size(ctypes.byref(a))
    ws = None
    if ws_bytes:
        ws = torch.empty(ws_bytes, device=q.device, dtype=torch.uint8)
        a.workspace, a.workspace_bytes = ws.data_ptr(), ws_bytes
    check(lib.poly_pass_bwd(ctypes.byref(a), _stream(q.device)), "poly_pass_bwd")
    del keep
    return dq, dk, dv, dbias


@torch.compiler.disable
def kernel_names(q, k, v, *, causal=False, bias=None, key_mask=None, query_mask=None):
    """(forward, backward) kernel family the library picks for these inputs."""
    a = PolyPassBwdArgs()
    out = torch.empty_like(q)
    lse = torch.empty(q.shape[:3], device=q.device, dtype=torch.float32)
    keep = []
    _fill_pass(a.fwd, q, k, v, out, lse, causal=causal, softclamp=None, scale=None, bias=bias, key_mask=key_mask,
               query_mask=query_mask, epi_mul=None, epi_out=None, keep=keep)
    g = [torch.empty_like(t, memory_format=torch.contiguous_format) for t in (q, q, k, v)]
    a.dout, a.dout_stride = g[0].data_ptr(), (g[0].stride(0), g[0].stride(1), g[0].stride(2))
    a.dq, a.dq_stride = g[1].data_ptr(), (g[1].stride(0), g[1].stride(1), g[1].stride(2))
    a.dk, a.dk_stride = g[2].data_ptr(), (g[2].stride(0), g[2].stride(1), g[2].stride(2))
    a.dv, a.dv_stride = g[3].data_ptr(), (g[3].stride(0), g[3].stride(1), g[3].stride(2))
    return (lib.poly_pass_fwd_kernel_name(ctypes.byref(a.fwd)).decode(),
            lib.poly_pass_bwd_kernel_name(ctypes.byref(a)).decode())


@torch.compiler.disable
def lse_merge(part_out, part_lse):
    """Merge key-split partials: part_out [P, ..., d], part_lse [P, ...] -> (out, lse)."""
    _require_cuda(part_out, part_lse)
    part_out = part_out.contiguous()
    part_lse = part_lse.float().contiguous()
    P, d = part_out.shape[0], part_out.shape[-1]
    out = torch.empty(part_out.shape[1:], device=part_out.device, dtype=part_out.dtype)
    lse = torch.empty(part_lse.shape[1:], device=part_out.device, dtype=torch.float32)
    a = PolyMergeArgs()
    a.parts, a.head_dim, a.dtype, a.rows = P, d, _DTYPES[part_out.dtype], part_lse[0].numel()
    a.part_out, a.part_lse, a.out, a.lse = part_out.data_ptr(), part_lse.data_ptr(), out.data_ptr(), lse.data_ptr()
    check(lib.poly_lse_merge(ctypes.byref(a), _stream(part_out.device)), "poly_lse_merge")
    return out, lse
