"""Per-head RMSNorm of the query / key tensors (the modules' ``q_norms``,
poly_attention/poly_attention.py:272, n_poly_attention.py:186-187) through
``poly_head_rmsnorm``: read straight from the strided head-split view, all
tensors of a layer in one launch, output contiguous.

Same results as ``nn.RMSNorm`` applied to each tensor: fp32 arithmetic, eps =
the module's eps or, if None, finfo(input dtype).eps, output in the input's
dtype (also inside autocast, which leaves rms_norm alone, and with float32
weights on 16-bit inputs). Registered as a torch.library custom op with a
fake implementation and autograd (backward by the closed-form RMSNorm
gradient in PyTorch), so torch.compile sees one node.
"""
from __future__ import annotations

import ctypes
from typing import List

import torch

from . import _lib
from ._lib import PolyHeadNorm, check, lib
from .ops import _DTYPES, _stream


def _out_dtype(x, w, out_fp32):
    return torch.float32 if out_fp32 else x.dtype


def _head_rmsnorm_impl(xs, ws, eps, out_fp32):
    outs = [torch.empty(x.shape, device=x.device, dtype=_out_dtype(x, w, out_fp32)) for x, w in zip(xs, ws)]
    for g0 in range(0, len(xs), _lib.MAX_NORMS):
        idx = list(range(g0, min(len(xs), g0 + _lib.MAX_NORMS)))
        arr = (PolyHeadNorm * len(idx))()
        keep = []
        for a, i in zip(arr, idx):
            x, w, o = xs[i], ws[i], outs[i]
            if not w.is_contiguous() or w.data_ptr() % 16:      # the kernel reads weights as 16-byte vectors
                w = w.contiguous().clone()
                keep.append(w)
            b, h, n, d = x.shape
            a.src, a.dst, a.weight = x.data_ptr(), o.data_ptr(), w.data_ptr()
            a.batch, a.heads, a.rows, a.dim = b, h, n, d
            a.src_stride[0], a.src_stride[1], a.src_stride[2] = x.stride(0), x.stride(1), x.stride(2)
            a.src_dtype, a.dst_dtype, a.weight_dtype = _DTYPES[x.dtype], _DTYPES[o.dtype], _DTYPES[w.dtype]
            a.eps = eps[i]
        check(lib.poly_head_rmsnorm(arr, len(idx), _stream(xs[0].device)), "poly_head_rmsnorm")
    return outs


@torch.library.custom_op("poly_b200::head_rmsnorm", mutates_args=())
def _head_rmsnorm(xs: List[torch.Tensor], ws: List[torch.Tensor], eps: List[float],
                  out_fp32: bool) -> List[torch.Tensor]:
    return _head_rmsnorm_impl(xs, ws, eps, out_fp32)


@_head_rmsnorm.register_fake
def _(xs, ws, eps, out_fp32):
    return [x.new_empty(x.shape, dtype=_out_dtype(x, w, out_fp32)) for x, w in zip(xs, ws)]


def _setup(ctx, inputs, output):
    xs, ws, eps, out_fp32 = inputs
    ctx.n = len(xs)
    ctx.eps = eps
    ctx.save_for_backward(*xs, *ws)


def _backward(ctx, grads):
    n = ctx.n
    xs, ws = ctx.saved_tensors[:n], ctx.saved_tensors[n:]
    dxs, dws = [], []
    for x, w, g, e in zip(xs, ws, grads, ctx.eps):
        if g is None:
            dxs.append(None)
            dws.append(None)
            continue
        xf, gf, wf = x.float(), g.float(), w.float()
        rs = torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + e)
        xh = xf * rs
        gw = gf * wf
        dxs.append((rs * (gw - xh * (gw * xh).mean(-1, keepdim=True))).to(x.dtype))
        dws.append((gf * xh).reshape(-1, x.shape[-1]).sum(0).to(w.dtype))
    return dxs, dws, None, None


_head_rmsnorm.register_autograd(_backward, setup_context=_setup)


def head_rmsnorm(norms, xs):
    """Apply ``norms[i]`` (nn.RMSNorm over the last dim) to ``xs[i]`` ([b, h, n, d]
    views); CUDA tensors of one dtype go through the library in one launch."""
    usable = (all(x.is_cuda and x.dim() == 4 and x.dtype in _DTYPES and x.stride(-1) == 1 for x in xs) and
              all(nm.weight is not None and nm.weight.dtype in (x.dtype, torch.float32)
                  for nm, x in zip(norms, xs)) and len({x.dtype for x in xs}) == 1 and
              len({nm.weight.dtype for nm in norms}) == 1 and
              all(x.shape[-1] % 8 == 0 and x.shape[-1] <= 256 for x in xs))
    if not usable:
        return [nm(x) for nm, x in zip(norms, xs)]
    eps = [float(nm.eps) if nm.eps is not None else float(torch.finfo(xs[0].dtype).eps) for nm in norms]
    ws = [nm.weight for nm in norms]
    if not torch.compiler.is_compiling() and not (
            torch.is_grad_enabled() and any(t.requires_grad for t in (*xs, *ws))):
        # inference (e.g. a decoding step): no autograd or tracing to serve, so
        # the library call skips the custom-op dispatcher (~80 us of host time)
        return _head_rmsnorm_impl(list(xs), ws, eps, False)
    return list(_head_rmsnorm(list(xs), ws, eps, False))


__all__ = ["head_rmsnorm"]
