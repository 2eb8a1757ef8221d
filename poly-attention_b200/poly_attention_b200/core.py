"""Poly-attention cores built from the single-pass kernel.

* ``poly_attention_order2`` -- both passes of order-2 poly attention with
  autograd (the work of PolyFlashAttention,
  poly_attention/flash_poly_attention.py:319-446, and of
  reference_poly_attention, poly_attention/poly_attention.py:48-116).
* ``poly_attention_chain`` -- the order-n right-to-left chain
  (n_poly_attention.py:263-313) with autograd.
* ``flash_poly_attention`` -- the reference's function-level entry point
  (poly_attention/flash_poly_attention.py:448-456), same signature.

Key/value-side tensors (q2, q3, v3, ...) may carry fewer heads than q1
(grouped-query attention): every pass whose queries and keys are both
key/value tensors runs once per key/value head, and only the last pass reads
q1 at full head count. The reference repeats those tensors r times instead
(poly_attention/poly_attention.py:289-293); the results are identical.
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch

from .ops import pass_bwd, pass_fwd


def _exists(v):
    return v is not None


# The order-2 core is two torch.library custom ops (forward, backward) with a
# fake (shape) implementation and registered autograd, so torch.compile treats
# it as one opaque node (no graph break at the ctypes calls) and autocast
# regions work (inputs are cast to the autocast dtype first, as the
# reference's einsums are).

def _token_major(q):
    """Output buffer [b, h, n, d] laid out as [b, n, h, d] in memory, so that the
    modules' merge_heads ('b h n d -> b n (h d)', poly_attention.py:340) is a
    view instead of a copy."""
    b, h, n, d = q.shape
    return q.new_empty((b, n, h, d)).permute(0, 2, 1, 3)


def _dense(t):
    """t itself when every stride is positive (any layout the kernels read
    through strides, e.g. the token-major gradient of merge_heads), else a
    contiguous copy (broadcast gradients such as out.sum().backward())."""
    return t if all(st > 0 for st in t.stride()) else t.contiguous()


def _propagate_masks(cms):
    """Levels run from the last score to the first; once one level is masked,
    its lse (the next level's key bias) can hold fully excluded rows
    (-finfo.max), so every later level without a mask gets an all-true key
    mask: that routes it to the masked-pass kernels, which reproduce the
    reference's result for keys that are all dead."""
    cms = list(cms)
    seen = None
    for t in range(len(cms) - 1, -1, -1):
        if cms[t] is not None:
            seen = cms[t]
        elif seen is not None:
            cms[t] = torch.ones_like(seen, dtype=torch.bool)
    return tuple(cms)


def _sc(softclamp):
    return float(softclamp) if softclamp else 0.0


@torch.library.custom_op("poly_b200::order2_fwd", mutates_args=())
def _order2_fwd(q1: torch.Tensor, q2: torch.Tensor, q3: torch.Tensor, v3: torch.Tensor,
                q2_pass1: Optional[torch.Tensor], mask: Optional[torch.Tensor], cm1: Optional[torch.Tensor],
                cm2: Optional[torch.Tensor], softclamp: float, causal: bool
                ) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    """Both passes: returns (out, lse23, msg, lse12)."""
    sc = softclamp or None
    qp1 = q2 if q2_pass1 is None else q2_pass1
    # pass 1: q2 attends q3 (poly_attention/poly_attention.py:63-82)
    msg, lse23 = pass_fwd(qp1, q3, v3, causal=causal, softclamp=sc, key_mask=cm2)
    # pass 2: q1 attends q2 with lse23 as key bias (:91-114), written token-major
    out, lse12 = pass_fwd(q1, q2, msg, causal=causal, softclamp=sc, bias=lse23, key_mask=cm1, query_mask=mask,
                          out=_token_major(q1))
    return out, lse23, msg, lse12


@_order2_fwd.register_fake
def _(q1, q2, q3, v3, q2_pass1, mask, cm1, cm2, softclamp, causal):
    qp1 = q2 if q2_pass1 is None else q2_pass1
    f32 = torch.float32
    return (_token_major(q1), qp1.new_empty(qp1.shape[:3], dtype=f32),
            qp1.new_empty((*qp1.shape[:3], v3.shape[-1])), q1.new_empty(q1.shape[:3], dtype=f32))


@torch.library.custom_op("poly_b200::order2_bwd", mutates_args=())
def _order2_bwd(q1: torch.Tensor, q2: torch.Tensor, q3: torch.Tensor, v3: torch.Tensor,
                q2_pass1: Optional[torch.Tensor], mask: Optional[torch.Tensor], cm1: Optional[torch.Tensor],
                cm2: Optional[torch.Tensor], msg: torch.Tensor, lse23: torch.Tensor, out: torch.Tensor,
                lse12: torch.Tensor, dout: torch.Tensor, softclamp: float, causal: bool
                ) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    """Returns (dq1, dq2, dq3, dv3, dq2_pass1); dq2_pass1 is empty when q2_pass1 is None."""
    sc = softclamp or None
    # pass-2 backward: dq1, dq2 (as keys), dmsg (as values), dlse23 (key-bias grad)
    dq1, dq2_keys, dmsg, dlse23 = pass_bwd(q1, q2, msg, out, lse12, dout, causal=causal, softclamp=sc,
                                           bias=lse23, key_mask=cm1, query_mask=mask, want_dbias=True)
    # pass-1 backward with the log-sum-exp gradient folded in; dq2 parts summed in-kernel
    if q2_pass1 is None:
        dq2, dq3, dv3, _ = pass_bwd(q2, q3, v3, msg, lse23, dmsg, causal=causal, softclamp=sc, key_mask=cm2,
                                    dlse=dlse23, dq=dq2_keys, dq_accumulate=True)
        return dq1, dq2, dq3, dv3, q2.new_empty(0)
    dqp1, dq3, dv3, _ = pass_bwd(q2_pass1, q3, v3, msg, lse23, dmsg, causal=causal, softclamp=sc, key_mask=cm2,
                                 dlse=dlse23)
    return dq1, dq2_keys, dq3, dv3, dqp1


@_order2_bwd.register_fake
def _(q1, q2, q3, v3, q2_pass1, mask, cm1, cm2, msg, lse23, out, lse12, dout, softclamp, causal):
    dqp1 = q2.new_empty(0) if q2_pass1 is None else q2_pass1.new_empty(q2_pass1.shape)
    return (q1.new_empty(q1.shape), q2.new_empty(q2.shape), q3.new_empty(q3.shape), v3.new_empty(v3.shape), dqp1)


def _order2_setup(ctx, inputs, output):
    q1, q2, q3, v3, q2_pass1, mask, cm1, cm2, softclamp, causal = inputs
    out, lse23, msg, lse12 = output
    ctx.save_for_backward(q1, q2, q3, v3, q2_pass1, mask, cm1, cm2, msg, lse23, out, lse12)
    ctx.softclamp, ctx.causal = softclamp, causal
    ctx.mark_non_differentiable(lse23, msg, lse12)


def _order2_backward(ctx, dout, _dlse23, _dmsg, _dlse12):
    q1, q2, q3, v3, q2_pass1, mask, cm1, cm2, msg, lse23, out, lse12 = ctx.saved_tensors
    dq1, dq2, dq3, dv3, dqp1 = _order2_bwd(q1, q2, q3, v3, q2_pass1, mask, cm1, cm2, msg, lse23, out, lse12,
                                           _dense(dout), ctx.softclamp, ctx.causal)
    return dq1, dq2, dq3, dv3, (dqp1 if q2_pass1 is not None else None), None, None, None, None, None


_order2_fwd.register_autograd(_order2_backward, setup_context=_order2_setup)


def _autocast(*ts):
    """Inside a CUDA autocast region, cast the floating inputs of the attention
    core to the autocast dtype (the reference's einsums run in it there)."""
    if not torch.is_autocast_enabled("cuda"):
        return ts
    dt = torch.get_autocast_dtype("cuda")
    return tuple(t.to(dt) if t is not None and t.is_floating_point() and t.dtype != dt else t for t in ts)


def poly_attention_order2(q1, q2, q3, v3, *, q2_pass1=None, mask=None, context_mask=None, softclamp_value=None,
                          causal=False):
    """Order-2 poly attention without cache. Returns (out, lse23, msg).

    q1 [b, h, n, d]; q2, q3, v3 [b, g, nk, d] (g divides h). ``q2_pass1``
    (default q2) is pass 1's query; ``mask`` masks queries of pass 2 and
    ``context_mask = (cm1, cm2)`` masks keys of pass 2 / pass 1, exactly as in
    reference_poly_attention. lse23 / msg are at g heads.
    """
    cm1, cm2 = context_mask if _exists(context_mask) else (None, None)
    cm1, cm2 = _propagate_masks((cm1, cm2))
    q1, q2, q3, v3, q2_pass1 = _autocast(q1, q2, q3, v3, q2_pass1)
    out, lse23, msg, _ = _order2_fwd(q1, q2, q3, v3, q2_pass1, mask, cm1, cm2, _sc(softclamp_value), bool(causal))
    return out, lse23, msg


@torch.compiler.disable
def poly_attention_order2_cached(q1, q2_new, q2_full, q3_full, v3_full, lse_cache, msg_cache, *,
                                 softclamp_value=None, context_mask=None, mask=None):
    """One KV-cache step of order 2 (poly_attention/poly_attention.py:84-87,
    283-287): pass 1 for the new rows against the full cache, then pass 2 of
    q1 against q2_full with the concatenated (lse23, msg). No causal mask, as
    in the reference when a cache is given. Returns (out, lse23_step, msg_step).
    """
    cm1, cm2 = _propagate_masks(context_mask) if _exists(context_mask) else (None, None)
    msg_step, lse_step = pass_fwd(q2_new, q3_full, v3_full, softclamp=softclamp_value, key_mask=cm2)
    lse = lse_step if lse_cache is None else torch.cat((lse_cache.float(), lse_step), -1)
    msg = msg_step if msg_cache is None else torch.cat((msg_cache, msg_step), -2)
    out, _ = pass_fwd(q1, q2_full, msg, softclamp=softclamp_value, bias=lse, key_mask=cm1, query_mask=mask)
    return out, lse_step, msg_step


class _Chain(torch.autograd.Function):
    """Order-n chain. Inputs: order query tensors ``ql`` (queries of each
    score), order key tensors ``qr`` and order-1 value tensors ``vs``."""

    @staticmethod
    def forward(ctx, order, softclamp, causal, mask, cms, *tensors):
        ql = list(tensors[:order])
        qr = list(tensors[order:2 * order])
        vs = list(tensors[2 * order:])
        vals, biases, msgs, lses, outs = [None] * order, [None] * order, [None] * order, [None] * order, [None] * order
        val, bias = vs[-1], None
        for t in range(order - 1, 0, -1):
            vals[t], biases[t] = val, bias
            if t >= 2:
                # V' = v * msg fused into the epilogue (n_poly_attention.py:287)
                msg, lse, nxt = pass_fwd(ql[t], qr[t], val, causal=causal, softclamp=softclamp, bias=bias,
                                         key_mask=cms[t], epi_mul=vs[t - 2])
            else:
                msg, lse = pass_fwd(ql[t], qr[t], val, causal=causal, softclamp=softclamp, bias=bias,
                                    key_mask=cms[t])
                nxt = msg
            msgs[t], lses[t] = msg, lse
            val, bias = nxt, lse
        vals[0], biases[0] = val, bias
        out, lse0 = pass_fwd(ql[0], qr[0], val, causal=causal, softclamp=softclamp, bias=bias, key_mask=cms[0],
                             query_mask=mask, out=_token_major(ql[0]))
        outs[0], lses[0] = out, lse0
        ctx.order, ctx.softclamp, ctx.causal = order, softclamp, causal
        ctx.cms, ctx.mask = cms, mask
        ctx.save_for_backward(*ql, *qr, *vs, *[v for v in vals], *[b if b is not None else torch.empty(0) for b in biases],
                              *[m if m is not None else torch.empty(0) for m in msgs], *lses, out)
        # caches in the reference's order (level order-1 first, level 1 last)
        new_lses = tuple(lses[t] for t in range(order - 1, 0, -1))
        new_msgs = tuple(msgs[t] for t in range(order - 1, 0, -1))
        ctx.mark_non_differentiable(*new_lses, *new_msgs)
        return (out, *new_lses, *new_msgs)

    @staticmethod
    def backward(ctx, dout, *_unused):
        n = ctx.order
        st = ctx.saved_tensors
        ql, qr, vs = list(st[:n]), list(st[n:2 * n]), list(st[2 * n:3 * n - 1])
        o = 3 * n - 1
        vals = list(st[o:o + n]); o += n
        biases = [b if b.numel() else None for b in st[o:o + n]]; o += n
        msgs = [m if m.numel() else None for m in st[o:o + n]]; o += n
        lses = list(st[o:o + n]); o += n
        outs = [st[o]] + [msgs[t] for t in range(1, n)]
        dql, dqr, dvs = [None] * n, [None] * n, [None] * (n - 1)
        g_out, g_lse = dout, None
        for t in range(n):
            dq, dk, dv, db = pass_bwd(ql[t], qr[t], vals[t], outs[t], lses[t], g_out, causal=ctx.causal,
                                      softclamp=ctx.softclamp, bias=biases[t], key_mask=ctx.cms[t],
                                      query_mask=ctx.mask if t == 0 else None, dlse=g_lse,
                                      want_dbias=t < n - 1)
            dql[t], dqr[t] = dq, dk
            if t == n - 1:
                dvs[-1] = dv
                break
            if t == 0:
                g_out = dv
            else:
                dvs[t - 1] = dv * msgs[t + 1]
                g_out = dv * vs[t - 1]
            g_lse = db
        return (None, None, None, None, None, *dql, *dqr, *dvs)


@torch.compiler.disable   # the chain / cached cores run eagerly under torch.compile
def poly_attention_chain(q_left, q_right, vs, *, softclamp_value=None, causal=False, mask=None, context_masks=None):
    """Order-n chain without cache (n = len(q_left)).

    q_left[0] = q1 [b, h, n, d]; q_left[t >= 1], q_right[t], vs[t] are
    key/value-side tensors [b, g, n, d]. Returns (out, lses, msgs) with lses /
    msgs in the reference's cache order.
    """
    order = len(q_left)
    cms = _propagate_masks(context_masks) if context_masks is not None else (None,) * order
    q_left, q_right, vs = list(_autocast(*q_left)), list(_autocast(*q_right)), list(_autocast(*vs))
    res = _Chain.apply(order, softclamp_value, bool(causal), mask, cms, *q_left, *q_right, *vs)
    return res[0], res[1:order], res[order:]


@torch.compiler.disable
def poly_attention_chain_cached(q_left, q_right_full, vs_full, cache_lses, cache_msgs, *, softclamp_value=None,
                                mask=None, context_masks=None):
    """One KV-cache step of the order-n chain (n_poly_attention.py:265-313).

    The values of level t >= 1 are vs_full[t-1] * msg_full of level t+1; the
    product is taken inside the kernel from the two cached tensors (v_mul), so
    no full-length V' is materialised. Returns (out, new_lse_steps,
    new_msg_steps) in the reference's cache order.
    """
    order = len(q_left)
    cms = _propagate_masks(context_masks) if context_masks is not None else (None,) * order
    val, vmul, bias = vs_full[-1], None, None
    step_lses, step_msgs = [], []
    for t in range(order - 1, 0, -1):
        idx = (order - 1) - t
        msg_step, lse_step = pass_fwd(q_left[t], q_right_full[t], val, softclamp=softclamp_value, bias=bias,
                                      key_mask=cms[t], v_mul=vmul)
        step_lses.append(lse_step)
        step_msgs.append(msg_step)
        lse_full = lse_step if cache_lses is None else torch.cat((cache_lses[idx].float(), lse_step), -1)
        msg_full = msg_step if cache_msgs is None else torch.cat((cache_msgs[idx], msg_step), -2)
        bias = lse_full
        if t >= 2:
            val, vmul = vs_full[t - 2], msg_full
        else:
            val, vmul = msg_full, None
    out, _ = pass_fwd(q_left[0], q_right_full[0], val, softclamp=softclamp_value, bias=bias, key_mask=cms[0],
                      query_mask=mask, v_mul=vmul)
    return out, step_lses, step_msgs


def flash_poly_attention(q1, q2, q3, v3, mask=None, context_mask=None, softclamp_value=None, is_causal=True):
    """Drop-in for poly_attention/flash_poly_attention.py:448-456.

    Same arguments and error behaviour: ``context_mask`` is rejected with the
    reference's AssertionError; ``mask`` [b, n] masks keys in both passes.
    q2 / q3 / v3 may have fewer heads than q1 (grouped-query attention).
    """
    assert not _exists(context_mask), 'context_mask is not supported in flash_poly_attention'
    cm = (mask, mask) if _exists(mask) else None
    out, _, _ = poly_attention_order2(q1, q2, q3, v3, context_mask=cm, softclamp_value=softclamp_value,
                                      causal=is_causal)
    return out
