"""Order-n poly-attention module, API- and state_dict-compatible with
``NPolyAttention`` (n_poly_attention.py:42-340). The right-to-left chain of
passes (:263-313) runs on the CUDA library, with grouped-query passes
computed once per key/value head.
"""
from __future__ import annotations

from functools import partial

import torch
from torch import Tensor, nn
from torch.nn import Module, RMSNorm

from .core import poly_attention_chain, poly_attention_chain_cached
from .head_norm import head_rmsnorm
from .kv_cache import ModuleKVCache, usable as _inplace_usable
from .poly_attention import _rotary, cast_tuple, default, exists, merge_heads, split_heads

LinearNoBias = partial(nn.Linear, bias=False)


class NPolyAttention(Module):
    def __init__(self, dim, order=3, heads=8, kv_heads=None, dim_head=64, causal=False, shared_kv=False,
                 softclamp_value=None, use_rotary_embed=False, prenorm=False, separate_context_norms=False,
                 multiply_root_value=False, use_root_value_as_attn_gate=False, attn_gate=False):
        super().__init__()
        assert order > 1, 'order must be greater than 1'
        self.norm = RMSNorm(dim) if prenorm else nn.Identity()
        self.context_norms = None
        if separate_context_norms and prenorm:
            self.context_norms = nn.ModuleList([RMSNorm(dim) for _ in range(order)])
        self.scale = dim_head ** -0.5
        kv_heads = default(kv_heads, heads)
        assert (heads % kv_heads) == 0, 'heads must be divisible by kv_heads'
        self.heads, self.kv_heads, self.dim_head = heads, kv_heads, dim_head
        self.causal, self.shared_kv, self.softclamp_value = causal, shared_kv, softclamp_value
        self.multiply_root_value = multiply_root_value
        self.use_root_value_as_attn_gate = use_root_value_as_attn_gate
        self.attn_gate = attn_gate
        self.is_gqa = heads != kv_heads
        assert not (use_root_value_as_attn_gate and (self.is_gqa or self.shared_kv)), \
            'cannot use root value as attention gate if using GQA or shared KV'
        self.q_split = 2 if attn_gate else 1
        self.has_root_v = multiply_root_value and not shared_kv
        self.kv1_split = 2 if self.has_root_v else 1
        self.kv_split = 1 if shared_kv else 2
        self.num_rep = heads // kv_heads
        self.order = order
        dim_inner, dim_inner_kv = dim_head * heads, dim_head * kv_heads
        self.to_q = LinearNoBias(dim, dim_inner * self.q_split)
        self.to_kvs = nn.ModuleList([
            LinearNoBias(dim, dim_inner_kv * self.kv1_split),
            *[LinearNoBias(dim, dim_inner_kv * (1 if shared_kv else 2)) for _ in range(order - 1)],
        ])
        self.q_norms = nn.ModuleList([RMSNorm(dim_head) for _ in range(order + 1)])
        self.rotary_emb = _rotary().RotaryEmbedding(dim_head) if use_rotary_embed else None
        self.to_out = nn.Linear(dim_inner, dim)
        # buffers behind the cache tuple returned last (in-place decoding steps)
        self._kv_cache = None

    def _expand(self, t):
        return t if (t is None or self.num_rep == 1) else t.repeat_interleave(self.num_rep, dim=1)

    def _finish(self, out, root_value, gates):
        """Root-value / attention gates, merge heads, output projection
        (n_poly_attention.py:315-328)."""
        if self.multiply_root_value:
            if self.use_root_value_as_attn_gate:
                root_value = root_value.sigmoid()
            out = self._expand(root_value) * out
        if self.attn_gate:
            out = out * gates.sigmoid()
        return self.to_out(merge_heads(out))

    def _squeeze(self, t):
        return t if (t is None or self.num_rep == 1) else t[:, ::self.num_rep]

    def forward(self, x, context: Tensor | tuple[Tensor, ...] | None = None, mask=None,
                context_mask: Tensor | tuple[Tensor | None, ...] | None = None, rotary_pos_emb=None, cache=None,
                return_cache=False):
        order = self.order
        seq_len = x.shape[-2]
        has_cache = exists(cache)
        if has_cache:
            assert seq_len == 1, 'sequence length must be 1 when using kv cache'
        orig_x = x
        x = self.norm(x)
        qg = split_heads(self.to_q(x), self.q_split, self.heads)
        q1 = qg[0]
        gates = qg[1] if self.attn_gate else None

        has_context = exists(context)
        context = cast_tuple(default(context, orig_x), order)
        assert len(context) == order
        if self.multiply_root_value:
            assert context[0].shape[-2] == seq_len, \
                'first context sequence length (context[0]) must match base sequence x when multiply_root_value is True'
        if exists(context_mask):
            context_mask = cast_tuple(context_mask, order)
            assert len(context_mask) == order
        elif not has_context and exists(mask):
            context_mask = (mask,) * order
        else:
            context_mask = (None,) * order
        if exists(self.context_norms):
            context = tuple(norm(c) for c, norm in zip(context, self.context_norms))
        else:
            context = context if has_context else (x,) * order

        kv1 = split_heads(self.to_kvs[0](context[0]), self.kv1_split, self.kv_heads)
        kvs_rest = [split_heads(to_kv(c), self.kv_split, self.kv_heads) for c, to_kv in zip(context[1:], self.to_kvs[1:])]
        qs_rest = (kv1[0], *[kv[0] for kv in kvs_rest])
        if self.shared_kv:
            root_value = qs_rest[0]
            vs = qs_rest[1:]
        else:
            vs = tuple(kv[1] for kv in kvs_rest)
            root_value = kv1[1] if self.has_root_v else None
        qs = tuple(head_rmsnorm(self.q_norms, (q1, *qs_rest)))
        if exists(rotary_pos_emb):
            r = _rotary()
            qs = tuple(r.apply_rotary_emb(rotary_pos_emb, q) for q in qs)
        q1, qs_rest = qs[0], qs[1:]

        inplace = (_inplace_usable(q1.dtype, q1.device, self.dim_head, exists(mask) or any(exists(m) for m in context_mask),
                                   exists(rotary_pos_emb) or exists(self.rotary_emb))
                   and (not has_cache or all(torch.is_tensor(t) and t.dtype == q1.dtype
                                             for part in cache for t in part)))
        if has_cache and inplace:
            # append in place to the module's cache buffers (a copy first if
            # the tuple is not the one this module returned last)
            c_qs, c_vs, c_lses, c_msgs = cache
            kv = self._kv_cache
            if kv is None or (cache is not kv.last and not kv.owns(list(c_qs), list(c_vs), list(c_lses), list(c_msgs))):
                kv = ModuleKVCache.from_tuple(list(c_qs), list(c_vs), list(c_lses), list(c_msgs), heads=self.heads,
                                              softclamp_value=self.softclamp_value)
            if kv.length >= kv.cap:
                kv = kv.grown()
            self._kv_cache = kv
            out = self._finish(kv.step(q1, list(qs_rest), list(vs)), root_value, gates)
            if not return_cache:
                return out
            k, v, l, m = kv.views()
            return out, kv.remember((tuple(k), tuple(v), tuple(l), tuple(m)))
        if has_cache:
            c_qs, c_vs, c_lses, c_msgs = cache
        else:
            c_qs, c_vs, c_lses, c_msgs = (None,) * order, (None,) * (order - 1), None, None
        cat = lambda c, t: t if c is None else torch.cat((c, t), dim=-2)  # noqa: E731
        qs_rest_cache = tuple(cat(c, q) for c, q in zip(c_qs, qs_rest))
        vs_cache = tuple(cat(c, v) for c, v in zip(c_vs, vs))

        q_left = [q1, *qs_rest[:-1]]
        q_right = list(qs_rest_cache)
        if not exists(rotary_pos_emb) and exists(self.rotary_emb):
            rot = [self.rotary_emb.rotate_queries_with_cached_keys(ql, qr) for ql, qr in zip(q_left, q_right)]
            q_left, q_right = (list(t) for t in zip(*rot))

        if has_cache:
            out, lse_steps, msg_steps = poly_attention_chain_cached(
                q_left, q_right, list(vs_cache), [self._squeeze(t) for t in c_lses],
                [self._squeeze(t) for t in c_msgs], softclamp_value=self.softclamp_value, mask=mask,
                context_masks=context_mask)
        else:
            out, lse_steps, msg_steps = poly_attention_chain(
                q_left, q_right, list(vs_cache), softclamp_value=self.softclamp_value, causal=self.causal,
                mask=mask, context_masks=context_mask)

        out = self._finish(out, root_value, gates)
        if not return_cache:
            return out
        if inplace and not has_cache:
            # prefill: the returned cache lives in buffers later steps append to
            kv = ModuleKVCache.from_core(list(qs_rest_cache), list(vs_cache), list(lse_steps), list(msg_steps),
                                         heads=self.heads, softclamp_value=self.softclamp_value)
            self._kv_cache = kv
            k, v, l, m = kv.views()
            return out, kv.remember((tuple(k), tuple(v), tuple(l), tuple(m)))
        new_lses, new_msgs = [], []
        for i, (l, m) in enumerate(zip(lse_steps, msg_steps)):
            l = self._expand(l).to(out.dtype)
            m = self._expand(m)
            new_lses.append(l if c_lses is None else torch.cat((c_lses[i], l), dim=-1))
            new_msgs.append(m if c_msgs is None else torch.cat((c_msgs[i], m), dim=-2))
        return out, (qs_rest_cache, vs_cache, tuple(new_lses), tuple(new_msgs))
