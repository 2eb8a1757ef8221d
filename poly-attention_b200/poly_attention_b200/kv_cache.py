"""In-place KV cache behind the modules' returned cache tuples.

The reference grows every cache tensor with ``torch.cat`` on each decoding
step (poly_attention/poly_attention.py:283-287,357-365;
n_poly_attention.py:196-207,332-340), so a step copies the whole cache.
``ModuleKVCache`` keeps the same contents in buffers of a fixed capacity that
doubles when full (one copy per doubling), and the tuples a module returns
are views of the first ``length`` rows of those buffers. When a module is
handed back the tuple it returned last, the step appends one row in place
and runs the decode kernels (``ChainDecoder``); any other cache tuple (from
another module, an older step, a branch of the sequence) is first copied
into fresh buffers once, so results never depend on which path ran.

Layouts (the reference's): key / value caches ``[b, g, L, d]`` at kv-head
width; lse caches ``[b, h, L]`` in the output dtype and msg caches
``[b, h, L, d]``, every query head of a group holding its group's values.
The kernels read kv-head-width copies of lse (fp32) and msg, which the
decoder owns; the h-head tensors are mirrors kept for the returned tuple.
"""
from __future__ import annotations

import torch

from .decode import ChainDecoder


class ModuleKVCache:
    def __init__(self, *, batch, order, heads, kv_heads, dim_head, dtype, device, capacity, softclamp_value=None):
        self.b, self.order, self.h, self.g, self.d = batch, order, heads, kv_heads, dim_head
        self.r = heads // kv_heads
        self.dtype, self.device, self.cap = dtype, torch.device(device), capacity
        self.softclamp_value = softclamp_value
        self.dec = ChainDecoder(batch=batch, order=order, heads=heads, kv_heads=kv_heads, dim_head=dim_head,
                                capacity=capacity, dtype=dtype, device=device, softclamp_value=softclamp_value)
        self.api_lses = [torch.empty(batch, heads, capacity, device=device, dtype=dtype) for _ in range(order - 1)]
        self.api_msgs = [torch.empty(batch, heads, capacity, dim_head, device=device, dtype=dtype)
                         for _ in range(order - 1)]
        self.last = None   # the tuple object last returned for the current views

    @property
    def length(self):
        return self.dec.length

    # ------------------------------------------------------------------ views
    def views(self):
        """(keys, values, lses, msgs) of the first `length` rows, reference layout."""
        n = self.length
        return ([q[:, :, :n] for q in self.dec.qs], [v[:, :, :n] for v in self.dec.vs],
                [t[:, :, :n] for t in self.api_lses], [t[:, :, :n] for t in self.api_msgs])

    def owns(self, keys, vals, lses, msgs):
        """True if these tensors are exactly this cache's current views."""
        n = self.length
        mine = (self.dec.qs, self.dec.vs, self.api_lses, self.api_msgs)
        for given, bufs in zip((keys, vals, lses, msgs), mine):
            if len(given) != len(bufs):
                return False
            for t, buf in zip(given, bufs):
                if (not torch.is_tensor(t) or t.data_ptr() != buf.data_ptr() or t.dtype != buf.dtype
                        or t.dim() != buf.dim() or t.shape[2] != n or t.stride() != buf.stride()):
                    return False
        return True

    # ------------------------------------------------------------------ fills
    def _fill(self, keys, vals, lses_g, msgs_g, lses_api=None, msgs_api=None):
        n = keys[0].shape[2]
        if n > self.cap:
            raise ValueError("cache longer than the capacity")
        for buf, t in zip(self.dec.qs + self.dec.vs, list(keys) + list(vals)):
            buf[:, :, :n].copy_(t)
        for i in range(self.order - 1):
            self.dec.lses[i][:, :, :n].copy_(lses_g[i])
            self.dec.msgs[i][:, :, :n].copy_(msgs_g[i])
            if lses_api is not None:
                self.api_lses[i][:, :, :n].copy_(lses_api[i])
                self.api_msgs[i][:, :, :n].copy_(msgs_api[i])
            else:
                self._mirror(i, slice(0, n))
        self.dec.length = n

    def _mirror_pairs(self, i, rows):
        """(destination, source) of the h-head mirrors of level i's rows."""
        b, g, r = self.b, self.g, self.r
        lg, mg = self.dec.lses[i][:, :, rows], self.dec.msgs[i][:, :, rows]
        n = lg.shape[-1]
        return ((self.api_lses[i][:, :, rows].view(b, g, r, n), lg[:, :, None].expand(b, g, r, n)),
                (self.api_msgs[i][:, :, rows].view(b, g, r, n, self.d), mg[:, :, None].expand(b, g, r, n, self.d)))

    def _mirror(self, i, rows):
        for dst, src in self._mirror_pairs(i, rows):
            dst.copy_(src)

    @classmethod
    def from_core(cls, keys, vals, lses_g, msgs_g, *, heads, capacity=None, softclamp_value=None):
        """After a prefill: keys / values [b, g, n, d], the core's lse (fp32) and
        msg at kv-head width."""
        b, g, n, d = keys[0].shape
        cap = capacity or max(2 * n, n + 64)
        c = cls(batch=b, order=len(keys), heads=heads, kv_heads=g, dim_head=d, dtype=keys[0].dtype,
                device=keys[0].device, capacity=cap, softclamp_value=softclamp_value)
        c._fill(keys, vals, [t.float() for t in lses_g], msgs_g)
        return c

    @classmethod
    def from_tuple(cls, keys, vals, lses, msgs, *, heads, softclamp_value=None):
        """From cache tensors in the reference layout (lse / msg at h heads)."""
        b, g, n, d = keys[0].shape
        r = heads // g
        c = cls(batch=b, order=len(keys), heads=heads, kv_heads=g, dim_head=d, dtype=keys[0].dtype,
                device=keys[0].device, capacity=max(2 * n, n + 64), softclamp_value=softclamp_value)
        c._fill(keys, vals, [t[:, ::r].float() for t in lses], [t[:, ::r] for t in msgs],
                lses_api=lses, msgs_api=msgs)
        return c

    def grown(self):
        """A copy with twice the capacity (the contents move once)."""
        k, v, l_api, m_api = self.views()
        n = self.length
        c = ModuleKVCache(batch=self.b, order=self.order, heads=self.h, kv_heads=self.g, dim_head=self.d,
                          dtype=self.dtype, device=self.device, capacity=2 * self.cap,
                          softclamp_value=self.softclamp_value)
        c._fill(k, v, [t[:, :, :n] for t in self.dec.lses], [t[:, :, :n] for t in self.dec.msgs],
                lses_api=l_api, msgs_api=m_api)
        return c

    # ------------------------------------------------------------------ step
    def step(self, q1, keys_new, vals_new):
        """Append one row of every key / value cache in place and run the
        chain for it. q1 [b, h, 1, d]; keys_new / vals_new [b, g, 1, d].
        Returns out [b, h, 1, d]; the lse / msg rows land in the caches."""
        L = self.length
        self.dec.append_kv(keys_new, vals_new)
        out = self.dec.step(q1)
        pairs = [pr for i in range(self.order - 1) for pr in self._mirror_pairs(i, slice(L, L + 1))]
        torch._foreach_copy_([d for d, _ in pairs], [s_ for _, s_ in pairs])   # all mirror rows, few launches
        self.last = None
        return out

    def remember(self, cache):
        """Note the tuple object handed out for the current views (a cheap
        identity check for the next step; `owns` is the full check)."""
        self.last = cache
        return cache


def usable(dtype, device, dim_head, has_masks, has_rotary):
    """Whether a module's cache step can take the in-place path."""
    return (not has_masks and not has_rotary and device.type == "cuda"
            and dtype in (torch.float32, torch.float16, torch.bfloat16) and dim_head % 8 == 0)


__all__ = ["ModuleKVCache"]
