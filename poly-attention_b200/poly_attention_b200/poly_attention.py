"""Order-2 poly-attention module, API- and state_dict-compatible with
``Order2PolyAttention`` (poly_attention/poly_attention.py:120-365).

Projections, RMSNorms and gates are PyTorch (cuBLAS); the attention core is
the CUDA library, on every call (training, prefill and KV-cache steps).
"""
from __future__ import annotations

from functools import partial

import torch
from torch import Tensor, nn
from torch.nn import Module, RMSNorm

from .core import poly_attention_order2, poly_attention_order2_cached
from .head_norm import head_rmsnorm
from .kv_cache import ModuleKVCache, usable as _inplace_usable

LinearNoBias = partial(nn.Linear, bias=False)


def exists(v):
    return v is not None


def default(v, d):
    return v if exists(v) else d


def cast_tuple(t, length=1):
    return (t,) * length if torch.is_tensor(t) or not isinstance(t, tuple) else t


def split_heads(t, split, heads):
    """'b n (split h d) -> split b h n d' as strided views (no copy)."""
    b, n, f = t.shape
    d = f // (split * heads)
    return t.view(b, n, split, heads, d).permute(2, 0, 3, 1, 4)


def merge_heads(t):
    """'b h n d -> b n (h d)'."""
    b, h, n, d = t.shape
    return t.transpose(1, 2).reshape(b, n, h * d)


def _rotary():
    try:
        import rotary_embedding_torch as r
    except ImportError as e:  # pragma: no cover - depends on the environment
        raise ImportError("rotary embeddings need the rotary-embedding-torch package") from e
    return r


class Order2PolyAttention(Module):
    def __init__(self, dim, heads=8, kv_heads=None, dim_head=64, causal=False, shared_kv=False, softclamp_value=None,
                 use_rotary_embed=False, prenorm=False, separate_context_norms=False, multiply_root_value=False,
                 use_root_value_as_attn_gate=False, attn_gate=False, use_flash_kernel=None):
        super().__init__()
        # use_flash_kernel is accepted for API compatibility: the CUDA core is always used
        self.use_flash_kernel = True
        self.norm = RMSNorm(dim) if prenorm else nn.Identity()
        self.context_norms = None
        if separate_context_norms and prenorm:
            self.context_norms = nn.ModuleList([RMSNorm(dim), RMSNorm(dim)])
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
        dim_inner, dim_inner_kv = dim_head * heads, dim_head * kv_heads
        self.to_q = LinearNoBias(dim, dim_inner * self.q_split)
        self.to_kvs = nn.ModuleList([
            LinearNoBias(dim, dim_inner_kv * self.kv1_split),
            LinearNoBias(dim, dim_inner_kv * (1 if shared_kv else 2)),
        ])
        self.q_norms = nn.ModuleList([RMSNorm(dim_head), RMSNorm(dim_head), RMSNorm(dim_head)])
        self.rotary_emb = _rotary().RotaryEmbedding(dim_head) if use_rotary_embed else None
        self.to_out = nn.Linear(dim_inner, dim)
        # buffers behind the cache tuple returned last (in-place decoding steps)
        self._kv_cache = None

    def _finish(self, out, v2, gates):
        """Root-value / attention gates, merge heads, output projection
        (poly_attention/poly_attention.py:342-355)."""
        if self.multiply_root_value:
            if self.use_root_value_as_attn_gate:
                v2 = v2.sigmoid()
            out = self._expand(v2) * out
        if self.attn_gate:
            out = out * gates.sigmoid()
        return self.to_out(merge_heads(out))

    def _expand(self, t):
        # [b, g, ...] -> [b, h, ...] as 'b g ... -> b (g r) ...'
        return t if self.num_rep == 1 else t.repeat_interleave(self.num_rep, dim=1)

    def _squeeze(self, t):
        # inverse of _expand for per-group identical tensors
        return t if (t is None or self.num_rep == 1) else t[:, ::self.num_rep]

    def forward(self, x, context: Tensor | tuple[Tensor, ...] | None = None, mask=None,
                context_mask: Tensor | tuple[Tensor | None, ...] | None = None, rotary_pos_emb=None, cache=None,
                return_cache=False):
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
        context = cast_tuple(default(context, orig_x), 2)
        assert len(context) == 2
        if self.multiply_root_value:
            assert context[0].shape[-2] == seq_len, \
                'first context sequence length (context[0]) must match base sequence x when multiply_root_value is True'
        if exists(context_mask):
            context_mask = cast_tuple(context_mask, 2)
            assert len(context_mask) == 2
        elif not has_context and exists(mask):
            context_mask = (mask, mask)
        else:
            context_mask = (None, None)
        if exists(self.context_norms):
            ctx1, ctx2 = (norm(c) for c, norm in zip(context, self.context_norms))
        else:
            ctx1, ctx2 = context if has_context else (x, x)

        kv1 = split_heads(self.to_kvs[0](ctx1), self.kv1_split, self.kv_heads)
        kv2 = split_heads(self.to_kvs[1](ctx2), self.kv_split, self.kv_heads)
        if self.shared_kv:
            q2, q3 = kv1[0], kv2[0]
            v2, v3 = kv1[0], kv2[0]
        else:
            q2 = kv1[0]
            v2 = kv1[1] if self.has_root_v else None
            q3, v3 = kv2[0], kv2[1]
        q1, q2, q3 = head_rmsnorm(self.q_norms, (q1, q2, q3))
        if exists(rotary_pos_emb):
            r = _rotary()
            q1, q2, q3 = (r.apply_rotary_emb(rotary_pos_emb, q) for q in (q1, q2, q3))

        cq2, cq3, cv3, clse23, cmsg = cache if has_cache else (None,) * 5
        inplace = (_inplace_usable(q1.dtype, q1.device, self.dim_head,
                                   exists(mask) or any(exists(m) for m in context_mask),
                                   exists(rotary_pos_emb) or exists(self.rotary_emb))
                   and (not has_cache or all(torch.is_tensor(t) and t.dtype == q1.dtype for t in cache)))
        if has_cache and inplace:
            # append in place to the module's cache buffers (a copy first if
            # the tuple is not the one this module returned last)
            kv = self._kv_cache
            if kv is None or (cache is not kv.last and not kv.owns([cq2, cq3], [cv3], [clse23], [cmsg])):
                kv = ModuleKVCache.from_tuple([cq2, cq3], [cv3], [clse23], [cmsg], heads=self.heads,
                                              softclamp_value=self.softclamp_value)
            if kv.length >= kv.cap:
                kv = kv.grown()
            self._kv_cache = kv
            out = kv.step(q1, [q2, q3], [v3])
            out = self._finish(out, v2, gates)
            if not return_cache:
                return out
            k, v, l, m = kv.views()
            return out, kv.remember((k[0], k[1], v[0], l[0], m[0]))
        cat = lambda c, t: t if c is None else torch.cat((c, t), dim=-2)  # noqa: E731
        q2_cache, q3_cache, v3_cache = cat(cq2, q2), cat(cq3, q3), cat(cv3, v3)

        q2_left, q2_right, q3_full = q2, q2_cache, q3_cache
        q2_pass1 = None
        if not exists(rotary_pos_emb) and exists(self.rotary_emb):
            q1, q2_right = self.rotary_emb.rotate_queries_with_cached_keys(q1, q2_right)
            q2_left, q3_full = self.rotary_emb.rotate_queries_with_cached_keys(q2_left, q3_full)
            q2_pass1 = q2_left

        if has_cache:
            out, lse_step, msg_step = poly_attention_order2_cached(
                q1, q2_left, q2_right, q3_full, v3_cache, self._squeeze(clse23), self._squeeze(cmsg),
                softclamp_value=self.softclamp_value, context_mask=context_mask, mask=mask)
        else:
            out, lse_step, msg_step = poly_attention_order2(
                q1, q2_right, q3_full, v3_cache, q2_pass1=q2_pass1, mask=mask, context_mask=context_mask,
                softclamp_value=self.softclamp_value, causal=self.causal)

        out = self._finish(out, v2, gates)
        if not return_cache:
            return out
        if inplace and not has_cache:
            # prefill: the returned cache lives in buffers later steps append to
            kv = ModuleKVCache.from_core([q2_cache, q3_cache], [v3_cache], [lse_step], [msg_step], heads=self.heads,
                                         softclamp_value=self.softclamp_value)
            self._kv_cache = kv
            k, v, l, m = kv.views()
            return out, kv.remember((k[0], k[1], v[0], l[0], m[0]))
        lse_step = self._expand(lse_step).to(out.dtype)
        msg_step = self._expand(msg_step)
        lse23_full = lse_step if clse23 is None else torch.cat((clse23, lse_step), dim=-1)
        msg_full = msg_step if cmsg is None else torch.cat((cmsg, msg_step), dim=-2)
        return out, (q2_cache, q3_cache, v3_cache, lse23_full, msg_full)


PolyAttention = Order2PolyAttention
