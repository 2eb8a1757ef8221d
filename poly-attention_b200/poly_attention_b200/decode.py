"""Serving-side KV-cache decoding of the order-n poly-attention core.

The reference grows its cache with ``torch.cat`` every step
(poly_attention/poly_attention.py:283-287, n_poly_attention.py:206-207,
281-302), copying the whole cache each time. ``ChainDecoder`` keeps the same
cache contents in buffers allocated once with a fixed capacity and appends
each new row in place. A step is one ``poly_decode_chain`` call: one decode
kernel per level (seq_q == 1), each writing its output row straight into the
level's msg / lse cache, launched as programmatic dependents so that a level
streams its cache while the previous level drains (a level reads the
previous level's output only in the appended row, the chain's contract).
Dtypes / sizes the decode kernel does not take run level by level through
``poly_pass_fwd``. The argument blocks live in one array built once; only the
length and the row pointers change per step.

Cache layout (kv-head width, as the kernels read it):
  qs[t]   [b, g, cap, d]  for t = 0 .. order-1  (q2 .. q_{order+1})
  vs[t]   [b, g, cap, d]  for t = 0 .. order-2  (v3 .. v_{order+1})
  lses[t] [b, g, cap]     fp32, reference cache order (level order-1 first)
  msgs[t] [b, g, cap, d]
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib
from ._lib import PolyPassArgs, check, lib
from .ops import _DTYPES


def _st3(t):
    return (t.stride(0), t.stride(1), t.stride(2))


class ChainDecoder:
    def __init__(self, *, batch, order, heads, kv_heads, dim_head, capacity, dtype=torch.bfloat16, device="cuda",
                 softclamp_value=None):
        assert order >= 2 and heads % kv_heads == 0
        self.b, self.order, self.h, self.g, self.d, self.cap = batch, order, heads, kv_heads, dim_head, capacity
        self.dtype, self.device = dtype, torch.device(device)
        self.softclamp = float(softclamp_value) if softclamp_value else 0.0
        mk = lambda: torch.zeros(batch, kv_heads, capacity, dim_head, device=device, dtype=dtype)  # noqa: E731
        self.qs = [mk() for _ in range(order)]
        self.vs = [mk() for _ in range(order - 1)]
        self.msgs = [mk() for _ in range(order - 1)]
        self.lses = [torch.zeros(batch, kv_heads, capacity, device=device, dtype=torch.float32)
                     for _ in range(order - 1)]
        self.length = 0
        self._stream = None
        # row copies of append_kv: one per key / value cache, fixed shape and strides
        nb = len(self.qs) + len(self.vs)
        self._copies = (_lib.PolyRowCopy * max(nb, 1))()
        for c, buf in zip(self._copies, self.qs + self.vs):
            esz = buf.element_size()
            c.outer, c.inner, c.row_bytes = batch, kv_heads, dim_head * esz
            c.dst_stride[0], c.dst_stride[1] = buf.stride(0) * esz, buf.stride(1) * esz
        # one argument block per level t = order-1 .. 0 (level t: queries q_{t+1}, keys q_{t+2}),
        # in launch order in one array (element order-1-t is level t)
        self._arr = (PolyPassArgs * order)()
        self._args = {}
        self._ws = {}
        self._chain = None           # poly_decode_chain usable (decided on the first step)
        self._ws_ready = False
        for t in range(order - 1, -1, -1):
            a = self._arr[order - 1 - t]
            a.batch, a.kv_heads, a.head_dim = batch, kv_heads, dim_head
            a.heads = heads if t == 0 else kv_heads
            a.seq_q = 1
            a.dtype = _DTYPES[dtype]
            a.causal = 0
            a.scale = dim_head ** -0.5
            a.softclamp = self.softclamp
            k = self.qs[t]
            a.k, a.k_stride = k.data_ptr(), _st3(k)
            if t == order - 1:
                v = self.vs[-1]
                a.v, a.v_stride = v.data_ptr(), _st3(v)
            elif t >= 1:
                v, vm = self.vs[t - 1], self.msgs[(order - 1) - (t + 1)]
                a.v, a.v_stride = v.data_ptr(), _st3(v)
                a.v_mul, a.v_mul_stride = vm.data_ptr(), _st3(vm)
            else:
                v = self.msgs[order - 2]
                a.v, a.v_stride = v.data_ptr(), _st3(v)
            if t < order - 1:
                bias = self.lses[(order - 1) - (t + 1)]
                a.bias, a.bias_stride = bias.data_ptr(), (bias.stride(0), bias.stride(1))
            if t >= 1:
                q = self.qs[t - 1]                       # the new row of q_{t+1}
                a.q_stride = _st3(q)
                msg, lse = self.msgs[(order - 1) - t], self.lses[(order - 1) - t]
                a.out_stride = _st3(msg)
                a.lse_stride = (lse.stride(0), lse.stride(1))
            self._args[t] = a

    def _workspace(self, t, a):
        need = lib.poly_pass_fwd_workspace_size(ctypes.byref(a))
        ws = self._ws.get(t)
        if ws is None or ws.numel() < need:
            ws = torch.empty(max(need, 1) * 2, device=self.device, dtype=torch.uint8)
            self._ws[t] = ws
        a.workspace, a.workspace_bytes = ws.data_ptr(), ws.numel()

    def append_kv(self, qs_new, vs_new):
        """Write one new row of every key / value tensor at position `length`."""
        L = self.length
        if L >= self.cap:
            raise ValueError("KV cache capacity exceeded")
        bufs, srcs = self.qs + self.vs, list(qs_new) + list(vs_new)
        if len(bufs) <= _lib.MAX_ROW_COPIES and all(x.is_cuda and x.dtype == self.dtype for x in srcs):
            esz = bufs[0].element_size()
            cps = self._copies
            for c, buf, x in zip(cps, bufs, srcs):
                c.src = x.data_ptr()
                c.src_stride[0], c.src_stride[1] = x.stride(0) * esz, x.stride(1) * esz
                c.dst = buf.data_ptr() + L * buf.stride(2) * esz
            stream = ctypes.c_void_p(torch.cuda.current_stream(self.device).cuda_stream)
            if lib.poly_copy_rows(cps, len(bufs), stream) == _lib.POLY_OK:   # one launch for every cache
                return
        dst = [buf[:, :, L:L + 1] for buf in bufs]
        torch._foreach_copy_(dst, srcs)

    def step(self, q1_new, out=None):
        """Run the chain for the row appended last; returns out [b, h, 1, d]."""
        L = self.length
        n = L + 1
        stream = ctypes.c_void_p(torch.cuda.current_stream(self.device).cuda_stream)
        if out is None:
            out = torch.empty(self.b, self.h, 1, self.d, device=self.device, dtype=self.dtype)
        esz = 4 if self.dtype == torch.float32 else 2
        for t in range(self.order - 1, -1, -1):
            a = self._args[t]
            a.seq_k = n
            if t >= 1:
                q = self.qs[t - 1]
                a.q = q.data_ptr() + L * q.stride(2) * esz
                msg, lse = self.msgs[(self.order - 1) - t], self.lses[(self.order - 1) - t]
                a.out = msg.data_ptr() + L * msg.stride(2) * esz
                a.lse = lse.data_ptr() + L * 4
            else:
                a.q, a.q_stride = q1_new.data_ptr(), _st3(q1_new)
                a.out, a.out_stride = out.data_ptr(), _st3(out)
                a.lse = None
        if not self._ws_ready:
            # few (batch, kv head) groups take the global-split decode, which
            # needs a workspace; size it once for the full capacity (the largest need)
            for t in range(self.order - 1, -1, -1):
                a = self._args[t]
                a.seq_k = self.cap
                self._workspace(t, a)
                a.seq_k = n
            self._ws_ready = True
        if self._chain is not False:
            rc = lib.poly_decode_chain(self._arr, self.order, stream)
            if rc == _lib.POLY_OK:
                self._chain = True
                self.length = n
                return out
            if rc != _lib.POLY_EUNSUPPORTED or self._chain:
                check(rc, "poly_decode_chain")
            self._chain = False
        for t in range(self.order - 1, -1, -1):
            a = self._args[t]
            self._workspace(t, a)
            check(lib.poly_pass_fwd(ctypes.byref(a), stream), "poly_pass_fwd (decode)")
        self.length = n
        return out

    def bytes_per_step(self):
        """Algorithmic HBM bytes the last step's kernels read (caches at kv-head width)."""
        n, b, g, d = self.length, self.b, self.g, self.d
        esz = 2 if self.dtype != torch.float32 else 4
        rows = (2 * self.order + (self.order - 1) - 1) * g * d * esz + (self.order - 1) * g * 4
        return b * n * rows


__all__ = ["ChainDecoder"]
_ = _lib
