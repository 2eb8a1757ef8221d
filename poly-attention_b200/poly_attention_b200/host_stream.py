"""Order-2 poly-attention training step on host tensors, streamed.

A caller whose q1 / q2 / q3 / v3 / dout live in host memory (a data loader's
pinned buffers, an FFI host) and who wants the gradients back in host memory
pays two PCIe transfers per step; done one after the other around the
kernels, they take longer than the kernels (at config 2: 335 MB in, 268 MB
out, ~3.8 ms of kernels). ``HostStreamedOrder2`` cuts the batch into chunks
and runs three CUDA streams over a ring of device slots: chunk c + 1 is copied
in while chunk c computes and chunk c - 1's gradients are copied out, so the
step costs about the slowest of the three (host-to-device bandwidth at
config 2) instead of their sum. Each chunk runs the same passes as
``poly_attention_order2``'s forward and backward (both causal passes of the
reference's ``reference_poly_attention``, poly_attention/poly_attention.py:48-116,
and their backward, flash_poly_attention.py:409-444); (batch, head) units are
independent, so chunking changes no result beyond fp32 summation order in
the dQ reduction.
"""
from __future__ import annotations

import torch

from .ops import pass_bwd, pass_fwd


class HostStreamedOrder2:
    def __init__(self, *, batch, heads, kv_heads, seq_len, dim_head, dtype=torch.bfloat16, device="cuda",
                 chunk=1, slots=3, causal=True, softclamp_value=None):
        if batch % chunk:
            raise ValueError("chunk must divide batch")
        if heads % kv_heads:
            raise ValueError("kv_heads must divide heads")
        self.b, self.h, self.g, self.n, self.d = batch, heads, kv_heads, seq_len, dim_head
        self.chunk, self.slots = chunk, slots
        self.causal, self.softclamp = bool(causal), softclamp_value
        self.device = torch.device(device)
        self.dtype = dtype
        shp_q = (chunk, heads, seq_len, dim_head)
        shp_k = (chunk, kv_heads, seq_len, dim_head)
        mk = lambda s: torch.empty(s, device=self.device, dtype=dtype)  # noqa: E731
        # slot s: (q1, q2, q3, v3, dout) of one chunk
        self._in = [[mk(shp_q), mk(shp_k), mk(shp_k), mk(shp_k), mk(shp_q)] for _ in range(slots)]
        self._s_h2d = torch.cuda.Stream(self.device)
        self._s_comp = torch.cuda.Stream(self.device)
        self._s_d2h = torch.cuda.Stream(self.device)
        self._in_ready = [torch.cuda.Event() for _ in range(slots)]
        self._in_free = [torch.cuda.Event() for _ in range(slots)]
        self._used = [False] * slots   # slot k has an earlier chunk whose compute must finish first
        self._next = 0                 # next slot (continues across steps)

    def _compute(self, q1, q2, q3, v3, do):
        sc, causal = self.softclamp, self.causal
        msg, lse23 = pass_fwd(q2, q3, v3, causal=causal, softclamp=sc)
        out, lse12 = pass_fwd(q1, q2, msg, causal=causal, softclamp=sc, bias=lse23)
        dq1, dq2, dmsg, dlse23 = pass_bwd(q1, q2, msg, out, lse12, do, causal=causal, softclamp=sc, bias=lse23,
                                          want_dbias=True)
        _, dq3, dv3, _ = pass_bwd(q2, q3, v3, msg, lse23, dmsg, causal=causal, softclamp=sc, dlse=dlse23, dq=dq2,
                                  dq_accumulate=True)
        return out, (dq1, dq2, dq3, dv3)

    def step(self, q1, q2, q3, v3, dout, grads=None, out=None, sync=True):
        """One forward + backward. Inputs: host tensors [b, h|g, n, d] (pinned
        for overlap). Gradients (dq1, dq2, dq3, dv3) are written into `grads`
        (host tensors, allocated pinned if None) and, if `out` is given, the
        forward output into it. Work is enqueued after everything already on
        the current stream. With sync=True the current stream then waits for
        the step, so events / synchronisation on it cover the whole step. With
        sync=False it does not: the next step's copies in start while this
        step's last chunks compute and copy out (steps overlap like a
        prefetching loader); call join() before reading the outputs."""
        hosts = (q1, q2, q3, v3, dout)
        for x in hosts:
            if x.is_cuda:
                raise ValueError("HostStreamedOrder2.step takes host tensors")
        if grads is None:
            grads = [torch.empty(x.shape, dtype=self.dtype, pin_memory=True) for x in (q1, q2, q3, v3)]
        cur = torch.cuda.current_stream(self.device)
        for s in (self._s_h2d, self._s_comp, self._s_d2h):
            s.wait_stream(cur)
        C = self.chunk
        for c in range(self.b // C):
            k = self._next
            self._next = (self._next + 1) % self.slots
            sl = slice(c * C, (c + 1) * C)
            with torch.cuda.stream(self._s_h2d):
                if self._used[k]:
                    self._s_h2d.wait_event(self._in_free[k])
                self._used[k] = True
                for dst, src in zip(self._in[k], hosts):
                    dst.copy_(src[sl], non_blocking=True)
                self._in_ready[k].record(self._s_h2d)
            with torch.cuda.stream(self._s_comp):
                self._s_comp.wait_event(self._in_ready[k])
                o, gs = self._compute(*self._in[k])
                self._in_free[k].record(self._s_comp)
            self._s_d2h.wait_stream(self._s_comp)
            with torch.cuda.stream(self._s_d2h):
                for dst, src in zip(grads, gs):
                    dst[sl].copy_(src, non_blocking=True)
                    src.record_stream(self._s_d2h)
                if out is not None:
                    out[sl].copy_(o, non_blocking=True)
                    o.record_stream(self._s_d2h)
        if sync:
            self.join()
        return grads

    def join(self):
        """Make the current stream wait for every step enqueued so far."""
        cur = torch.cuda.current_stream(self.device)
        cur.wait_stream(self._s_d2h)
        cur.wait_stream(self._s_h2d)

    def bytes_per_step(self):
        """(host-to-device, device-to-host) bytes of one step (gradients only)."""
        esz = torch.empty((), dtype=self.dtype).element_size()
        q, kv = self.b * self.h * self.n * self.d * esz, self.b * self.g * self.n * self.d * esz
        return 2 * q + 3 * kv, q + 3 * kv


__all__ = ["HostStreamedOrder2"]
