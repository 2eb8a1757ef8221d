"""CPU oracle for the poly-attention hot path (numpy restatement).

TEST INFRASTRUCTURE ONLY. This module is the checker the parity tests, the
``smoke()`` entry and the ``cpu_baseline`` / ``--impl reference`` legs of
``bench.py`` compare against. The product path (``poly_attention_b200``) never
imports it: the CUDA library is the only implementation that ships.

It restates, in numpy, the reference PyTorch (non-Triton) algorithm of
lucidrains/poly-attention 0.3.6. Every function cites the reference lines it
follows. All score matrices are materialised (O(n^2) memory), exactly like the
reference, so it is meant for small and medium sizes.

Semantics that are reproduced on purpose (they matter for parity):

* masking writes ``-finfo(dtype).max`` (not ``-inf``), so a row whose entries
  are all masked becomes a *uniform* average over every key
  (poly_attention/poly_attention.py:68,73,76,102,105);
* the pass-1 log-sum-exp is added as a per-key bias *after* masking
  (poly_attention/poly_attention.py:109), so it also receives gradient from
  masked entries;
* causal masking is ``triu(1)`` on the (i, j) score matrix, i.e. top-left
  aligned, and is skipped whenever a cache is given
  (poly_attention/poly_attention.py:70-73,96-99).

Pinned against golden vectors produced by running the reference itself
(``tests/golden/make_golden.py``), see ``tests/test_oracle_golden.py``.
"""
from __future__ import annotations

import numpy as np

__all__ = [
    "softclamp",
    "rmsnorm",
    "pass_fwd",
    "order2_fwd",
    "order2_bwd",
    "npoly_chain_fwd",
    "npoly_chain_bwd",
    "order2_module_fwd",
    "npoly_module_fwd",
]


def _mask_value(dtype):
    # poly_attention/poly_attention.py:68 ; n_poly_attention.py:242
    return -np.finfo(dtype).max


def softclamp(x, c):
    """c * tanh(x / c)  (poly_attention/poly_attention.py:43-44)."""
    return c * np.tanh(x / c)


def _logsumexp(s):
    m = np.max(s, axis=-1, keepdims=True)
    with np.errstate(over="ignore", invalid="ignore"):
        r = m + np.log(np.sum(np.exp(s - m), axis=-1, keepdims=True))
    return r[..., 0]


def _softmax(s):
    m = np.max(s, axis=-1, keepdims=True)
    with np.errstate(over="ignore", invalid="ignore"):
        e = np.exp(s - m)
        return e / np.sum(e, axis=-1, keepdims=True)


def _scores(ql, qr, scale, softclamp_value):
    """scale * ql qr^T, then optional softclamp.

    poly_attention/poly_attention.py:63-66,91-94 ; n_poly_attention.py:237-240
    Returns (scores, tanh_or_None) so the backward can reuse tanh.
    """
    s = np.matmul(ql, np.swapaxes(qr, -1, -2)) * ql.dtype.type(scale)
    t = None
    if softclamp_value is not None:
        t = np.tanh(s / s.dtype.type(softclamp_value))
        s = s.dtype.type(softclamp_value) * t
    return s, t


def _keep_mask(shape, causal, key_mask, query_mask):
    """Boolean 'kept' mask of shape [b, 1|h, i, j] (True = not masked).

    causal: triu(1) top-left aligned  (poly_attention/poly_attention.py:70-73)
    key_mask 'b j'                     (poly_attention/poly_attention.py:75-76,101-102)
    query_mask 'b i'                   (poly_attention/poly_attention.py:104-105)
    """
    b, h, i, j = shape
    keep = np.ones((b, 1, i, j), dtype=bool)
    if causal:
        keep &= ~np.triu(np.ones((i, j), dtype=bool), 1)[None, None]
    if key_mask is not None:
        keep &= key_mask.astype(bool)[:, None, None, :]
    if query_mask is not None:
        keep &= query_mask.astype(bool)[:, None, :, None]
    return keep


def pass_fwd(q, k, v, *, scale=None, causal=False, softclamp_value=None,
             key_mask=None, query_mask=None, bias=None):
    """One flash pass of poly attention, materialised.

    Order of operations (poly_attention/poly_attention.py:63-82 for pass 1 and
    :91-114 for pass 2): scores -> softclamp -> causal -> key mask -> query
    mask -> + per-key bias -> logsumexp / softmax -> P @ V.

    q [b,h,i,d], k [b,h,j,d], v [b,h,j,dv], bias [b,h,j] or None.
    Returns (out [b,h,i,dv], lse [b,h,i]).
    """
    if scale is None:
        scale = q.shape[-1] ** -0.5
    s, _ = _scores(q, k, scale, softclamp_value)
    keep = _keep_mask(s.shape, causal, key_mask, query_mask)
    s = np.where(keep, s, _mask_value(s.dtype))
    if bias is not None:
        with np.errstate(over="ignore"):
            s = s + bias[..., None, :].astype(s.dtype)
    lse = _logsumexp(s)
    p = _softmax(s)
    out = np.matmul(p, v)
    return out, lse


def order2_fwd(q1, q2_pass1, q2_pass2, q3, v3, mask=None, context_mask=None,
               softclamp_value=None, causal=False, cache=None):
    """Restatement of ``reference_poly_attention``
    (poly_attention/poly_attention.py:48-116).

    Returns (out, lse23_step, msg_step) like the reference.
    ``cache`` is the reference tuple (cq2, cq3, cv3, clse23, cmsg); only its
    last two entries are read here, as in the reference (:84-87).
    """
    scale = q1.shape[-1] ** -0.5
    has_cache = cache is not None
    cm1, cm2 = context_mask if context_mask is not None else (None, None)

    # pass 1 (:63-82)
    msg_step, lse23_step = pass_fwd(
        q2_pass1, q3, v3, scale=scale, causal=causal and not has_cache,
        softclamp_value=softclamp_value, key_mask=cm2)

    # cache concat (:84-87)
    if has_cache:
        clse23, cmsg = cache[3], cache[4]
        lse23 = np.concatenate([clse23, lse23_step], axis=-1)
        msg = np.concatenate([cmsg, msg_step], axis=-2)
    else:
        lse23, msg = lse23_step, msg_step

    # pass 2 (:91-114)
    out, _ = pass_fwd(
        q1, q2_pass2, msg, scale=scale, causal=causal and not has_cache,
        softclamp_value=softclamp_value, key_mask=cm1, query_mask=mask,
        bias=lse23)
    return out, lse23_step, msg_step


def _pass_bwd(q, k, v, dout, *, scale, causal, softclamp_value, key_mask,
              query_mask, bias, dlse=None):
    """Analytic gradient of ``pass_fwd`` (what torch autograd computes for the
    reference's materialised pass).

    Returns (dq, dk, dv, dbias) where dbias is the column sum of dS over the
    query axis (the gradient that flows into the added per-key bias,
    poly_attention/poly_attention.py:109) and ``dlse`` is an optional upstream
    gradient on the returned log-sum-exp (grad of logsumexp = softmax).
    """
    s, t = _scores(q, k, scale, softclamp_value)
    keep = _keep_mask(s.shape, causal, key_mask, query_mask)
    s = np.where(keep, s, _mask_value(s.dtype))
    if bias is not None:
        with np.errstate(over="ignore"):
            s = s + bias[..., None, :].astype(s.dtype)
    p = _softmax(s)
    dp = np.matmul(dout, np.swapaxes(v, -1, -2))
    dv = np.matmul(np.swapaxes(p, -1, -2), dout)
    ds = p * (dp - np.sum(p * dp, axis=-1, keepdims=True))
    if dlse is not None:
        ds = ds + p * dlse[..., None]
    dbias = np.sum(ds, axis=-2)
    dz = np.where(keep, ds, 0)
    if t is not None:
        dz = dz * (1 - t * t)
    dq = np.matmul(dz, k) * scale
    dk = np.matmul(np.swapaxes(dz, -1, -2), q) * scale
    return dq, dk, dv, dbias


def order2_bwd(q1, q2_pass1, q2_pass2, q3, v3, dout, mask=None,
               context_mask=None, softclamp_value=None, causal=False):
    """Gradient of ``order2_fwd``'s ``out`` w.r.t. (q1, q2_pass1, q2_pass2, q3,
    v3), no cache. This is what autograd through
    poly_attention/poly_attention.py:48-116 produces.

    Chain: pass-2 backward gives dq1, dq2_pass2, dmsg and dlse23 (column sum of
    dS12); pass-1 backward takes dmsg as dO and dlse23 as the log-sum-exp
    gradient and gives dq2_pass1, dq3, dv3.
    """
    scale = q1.shape[-1] ** -0.5
    cm1, cm2 = context_mask if context_mask is not None else (None, None)
    msg, lse23 = pass_fwd(q2_pass1, q3, v3, scale=scale, causal=causal,
                          softclamp_value=softclamp_value, key_mask=cm2)
    dq1, dq2_pass2, dmsg, dlse23 = _pass_bwd(
        q1, q2_pass2, msg, dout, scale=scale, causal=causal,
        softclamp_value=softclamp_value, key_mask=cm1, query_mask=mask,
        bias=lse23)
    dq2_pass1, dq3, dv3, _ = _pass_bwd(
        q2_pass1, q3, v3, dmsg, scale=scale, causal=causal,
        softclamp_value=softclamp_value, key_mask=cm2, query_mask=None,
        bias=None, dlse=dlse23)
    return dq1, dq2_pass1, dq2_pass2, dq3, dv3


def npoly_chain_fwd(q_left, q_right, vs_full, *, causal=False,
                    softclamp_value=None, context_masks=None, mask=None,
                    cache_lses=None, cache_msgs=None):
    """Right-to-left order-n chain (n_poly_attention.py:233-313).

    q_left  : [q1, q2_left, ..., q_{n-1}_left]   (queries of each score)
    q_right : [q2_full, ..., q_n_full]           (keys of each score)
    vs_full : [v3_full, ..., v_n_full]           (order-1 value tensors)
    Scores t = 0..order-1 are scale * q_left[t] q_right[t]^T with softclamp,
    causal (skipped with cache), context mask on keys, query mask on t = 0
    (:233-261). Returns (out, new_lses, new_msgs) where the lists are in the
    reference's cache order (level order-1 first, level 1 last, :268-305).
    """
    order = len(q_left)
    scale = q_left[0].shape[-1] ** -0.5
    has_cache = cache_lses is not None
    context_masks = context_masks or (None,) * order
    c_lses = cache_lses or (None,) * (order - 1)
    c_msgs = cache_msgs or (None,) * (order - 1)

    scores = []
    keeps = []
    for idx in range(order):
        s, _ = _scores(q_left[idx], q_right[idx], scale, softclamp_value)
        keep = _keep_mask(s.shape, causal and not has_cache, context_masks[idx],
                          mask if idx == 0 else None)
        s = np.where(keep, s, _mask_value(s.dtype))
        scores.append(s)
        keeps.append(keep)

    out = vs_full[-1]
    cur = scores[-1]
    new_lses, new_msgs = [], []

    def cat(c, x, axis):
        return x if c is None else np.concatenate([c, x], axis=axis)

    for k in range(order - 1, 1, -1):
        lse_step = _logsumexp(cur)
        msg_step = np.matmul(_softmax(cur), out)
        idx = (order - 1) - k
        lse_full = cat(c_lses[idx], lse_step, -1)
        msg_full = cat(c_msgs[idx], msg_step, -2)
        new_msgs.append(msg_full)
        new_lses.append(lse_full)
        out = vs_full[k - 2] * msg_full
        with np.errstate(over="ignore"):
            cur = lse_full[..., None, :] + scores[k - 1]

    lse1_step = _logsumexp(cur)
    msg1_step = np.matmul(_softmax(cur), out)
    idx = order - 2
    lse1_full = cat(c_lses[idx], lse1_step, -1)
    msg1_full = cat(c_msgs[idx], msg1_step, -2)
    new_msgs.append(msg1_full)
    new_lses.append(lse1_full)
    with np.errstate(over="ignore"):
        s12 = lse1_full[..., None, :] + scores[0]
    out = np.matmul(_softmax(s12), msg1_full)
    return out, new_lses, new_msgs


def npoly_chain_bwd(q_left, q_right, vs_full, dout, *, causal=False,
                    softclamp_value=None, context_masks=None, mask=None):
    """Gradient of ``npoly_chain_fwd``'s ``out`` (no cache) w.r.t. every
    q_left[t], q_right[t] and vs_full[t]: autograd of
    n_poly_attention.py:233-313 written out.

    Levels run left to right in the backward: the last pass (t = 0) gives
    dq_left[0], dq_right[0], dmsg_1 and dlse_1; each earlier pass t takes
    (dmsg, dlse) of level t, splits dV' = dmsg into dv (times msg of level
    t+1) and dmsg of level t+1 (times v), and so on.
    """
    order = len(q_left)
    scale = q_left[0].shape[-1] ** -0.5
    context_masks = context_masks or (None,) * order
    # forward, keeping every level's (value, bias)
    vals = [None] * order      # V used by pass t
    biases = [None] * order    # per-key bias of pass t
    msgs = [None] * order      # output of pass t (t >= 1)
    out = vs_full[-1]
    bias = None
    for t in range(order - 1, 0, -1):
        vals[t], biases[t] = out, bias
        msg, lse = pass_fwd(q_left[t], q_right[t], out, scale=scale, causal=causal,
                            softclamp_value=softclamp_value,
                            key_mask=context_masks[t], bias=bias)
        msgs[t] = msg
        bias = lse
        out = vs_full[t - 2] * msg if t >= 2 else msg
    vals[0], biases[0] = out, bias

    dq_left = [None] * order
    dq_right = [None] * order
    dvs = [None] * (order - 1)
    g_out, g_lse = dout, None
    for t in range(order):
        dql, dqr, dval, dbias = _pass_bwd(
            q_left[t], q_right[t], vals[t], g_out, scale=scale, causal=causal,
            softclamp_value=softclamp_value, key_mask=context_masks[t],
            query_mask=mask if t == 0 else None, bias=biases[t], dlse=g_lse)
        dq_left[t], dq_right[t] = dql, dqr
        if t == order - 1:
            dvs[-1] = dval
            break
        # vals[t] = vs_full[t-1] * msgs[t+1]  for t >= 1 ; vals[0] = msgs[1]
        if t == 0:
            g_out = dval
        else:
            dvs[t - 1] = dval * msgs[t + 1]
            g_out = dval * vs_full[t - 1]
        g_lse = dbias
    return dq_left, dq_right, dvs


# ---------------------------------------------------------------------------
# module-level restatements (projections, q-norms, GQA, gates)
# ---------------------------------------------------------------------------

def rmsnorm(x, weight, eps=None):
    """torch.nn.RMSNorm with eps=None (finfo(dtype).eps), as used at
    poly_attention/poly_attention.py:139,196-200."""
    if eps is None:
        eps = np.finfo(x.dtype).eps
    r = 1.0 / np.sqrt(np.mean(x * x, axis=-1, keepdims=True) + x.dtype.type(eps))
    return (x * r) * weight


def _linear(x, w, b=None):
    y = x @ w.T
    return y + b if b is not None else y


def _split(t, split, heads):
    # 'b n (split h d) -> split b h n d'
    b, n, f = t.shape
    d = f // (split * heads)
    return t.reshape(b, n, split, heads, d).transpose(2, 0, 3, 1, 4)


def _repeat_kv(t, r):
    # 'b g n d -> b (g r) n d'
    return None if t is None else np.repeat(t, r, axis=1)


def _sigmoid(x):
    return 1.0 / (1.0 + np.exp(-x))


def order2_module_fwd(p, x, *, heads, kv_heads=None, causal=False,
                      shared_kv=False, softclamp_value=None, prenorm=False,
                      multiply_root_value=False,
                      use_root_value_as_attn_gate=False, attn_gate=False,
                      context=None, mask=None, context_mask=None, cache=None,
                      return_cache=False):
    """Restatement of ``Order2PolyAttention.forward``
    (poly_attention/poly_attention.py:206-365), without rotary and without
    ``separate_context_norms``. ``p`` maps state_dict names to arrays.
    """
    kv_heads = kv_heads or heads
    seq_len = x.shape[-2]
    has_cache = cache is not None
    orig_x = x
    if prenorm:
        x = rmsnorm(x, p["norm.weight"])
    qg = _split(_linear(x, p["to_q.weight"]), 2 if attn_gate else 1, heads)
    q1 = qg[0]
    gates = qg[1] if attn_gate else None

    has_context = context is not None
    if context is None:
        context = orig_x
    if not isinstance(context, tuple):
        context = (context, context)
    if context_mask is not None:
        if not isinstance(context_mask, tuple):
            context_mask = (context_mask, context_mask)
    elif not has_context and mask is not None:
        context_mask = (mask, mask)
    else:
        context_mask = (None, None)
    ctx1, ctx2 = context if has_context else (x, x)

    has_root_v = multiply_root_value and not shared_kv
    kv1 = _split(_linear(ctx1, p["to_kvs.0.weight"]), 2 if has_root_v else 1, kv_heads)
    kv2 = _split(_linear(ctx2, p["to_kvs.1.weight"]), 1 if shared_kv else 2, kv_heads)
    if shared_kv:
        q2, q3 = kv1[0], kv2[0]
        v2, v3 = kv1[0], kv2[0]
    else:
        q2 = kv1[0]
        v2 = kv1[1] if has_root_v else None
        q3, v3 = kv2[0], kv2[1]
    q1 = rmsnorm(q1, p["q_norms.0.weight"])
    q2 = rmsnorm(q2, p["q_norms.1.weight"])
    q3 = rmsnorm(q3, p["q_norms.2.weight"])

    if has_cache:
        cq2, cq3, cv3 = cache[0], cache[1], cache[2]
        q2_cache = np.concatenate([cq2, q2], -2)
        q3_cache = np.concatenate([cq3, q3], -2)
        v3_cache = np.concatenate([cv3, v3], -2)
    else:
        q2_cache, q3_cache, v3_cache = q2, q3, v3
    r = heads // kv_heads
    if r > 1:
        q2, q3, v2, v3 = (_repeat_kv(t, r) for t in (q2, q3, v2, v3))
        q2_full, q3_full, v3_full = (_repeat_kv(t, r) for t in (q2_cache, q3_cache, v3_cache))
    else:
        q2_full, q3_full, v3_full = q2_cache, q3_cache, v3_cache

    out, lse23_step, msg_step = order2_fwd(
        q1, q2, q2_full, q3_full, v3_full, mask=mask, context_mask=context_mask,
        softclamp_value=softclamp_value, causal=causal, cache=cache)
    if multiply_root_value:
        if use_root_value_as_attn_gate:
            v2 = _sigmoid(v2)
        out = v2 * out
    if attn_gate:
        out = out * _sigmoid(gates)
    b, h, n, d = out.shape
    out = _linear(out.transpose(0, 2, 1, 3).reshape(b, n, h * d),
                  p["to_out.weight"], p["to_out.bias"])
    if not return_cache:
        return out
    if has_cache:
        lse_full = np.concatenate([cache[3], lse23_step], -1)
        msg_full = np.concatenate([cache[4], msg_step], -2)
    else:
        lse_full, msg_full = lse23_step, msg_step
    return out, (q2_cache, q3_cache, v3_cache, lse_full, msg_full)


def npoly_module_fwd(p, x, *, order, heads, kv_heads=None, causal=False,
                     shared_kv=False, softclamp_value=None, prenorm=False,
                     multiply_root_value=False,
                     use_root_value_as_attn_gate=False, attn_gate=False,
                     context=None, mask=None, context_mask=None, cache=None,
                     return_cache=False):
    """Restatement of ``NPolyAttention.forward`` (n_poly_attention.py:122-340),
    without rotary and without ``separate_context_norms``."""
    kv_heads = kv_heads or heads
    has_cache = cache is not None
    orig_x = x
    if prenorm:
        x = rmsnorm(x, p["norm.weight"])
    qg = _split(_linear(x, p["to_q.weight"]), 2 if attn_gate else 1, heads)
    q1 = qg[0]
    gates = qg[1] if attn_gate else None

    has_context = context is not None
    if context is None:
        context = orig_x
    if not isinstance(context, tuple):
        context = (context,) * order
    if context_mask is not None:
        if not isinstance(context_mask, tuple):
            context_mask = (context_mask,) * order
    elif not has_context and mask is not None:
        context_mask = (mask,) * order
    else:
        context_mask = (None,) * order
    context = context if has_context else (x,) * order

    has_root_v = multiply_root_value and not shared_kv
    kv1 = _split(_linear(context[0], p["to_kvs.0.weight"]), 2 if has_root_v else 1, kv_heads)
    kvs_rest = [_split(_linear(c, p[f"to_kvs.{i + 1}.weight"]), 1 if shared_kv else 2, kv_heads)
                for i, c in enumerate(context[1:])]
    qs_rest = (kv1[0], *[kv[0] for kv in kvs_rest])
    if shared_kv:
        root_value = qs_rest[0]
        vs = qs_rest[1:]
    else:
        vs = tuple(kv[1] for kv in kvs_rest)
        root_value = kv1[1] if has_root_v else None
    qs = (q1, *qs_rest)
    qs = tuple(rmsnorm(q, p[f"q_norms.{i}.weight"]) for i, q in enumerate(qs))
    # with shared_kv the aggregation values are the *un-normed* projections
    # (n_poly_attention.py:177-180 bind them before the norms at :188)
    q1, qs_rest = qs[0], qs[1:]

    if has_cache:
        c_qs, c_vs, c_lses, c_msgs = cache
    else:
        c_qs = (None,) * order
        c_vs = (None,) * (order - 1)
        c_lses = c_msgs = None

    def cat(c, x_):
        return x_ if c is None else np.concatenate([c, x_], -2)

    qs_rest_cache = tuple(cat(c, q) for c, q in zip(c_qs, qs_rest))
    vs_cache = tuple(cat(c, v) for c, v in zip(c_vs, vs))
    r = heads // kv_heads
    if r > 1:
        qs_left = tuple(_repeat_kv(t, r) for t in qs_rest)
        qs_right = tuple(_repeat_kv(t, r) for t in qs_rest_cache)
        vs_full = tuple(_repeat_kv(t, r) for t in vs_cache)
        root_value = _repeat_kv(root_value, r)
    else:
        qs_left, qs_right, vs_full = qs_rest, qs_rest_cache, vs_cache

    out, new_lses, new_msgs = npoly_chain_fwd(
        [q1, *qs_left[:-1]], list(qs_right), list(vs_full), causal=causal,
        softclamp_value=softclamp_value, context_masks=context_mask, mask=mask,
        cache_lses=c_lses, cache_msgs=c_msgs)
    if multiply_root_value:
        if use_root_value_as_attn_gate:
            root_value = _sigmoid(root_value)
        out = root_value * out
    if attn_gate:
        out = out * _sigmoid(gates)
    b, h, n, d = out.shape
    out = _linear(out.transpose(0, 2, 1, 3).reshape(b, n, h * d),
                  p["to_out.weight"], p["to_out.bias"])
    if not return_cache:
        return out
    return out, (qs_rest_cache, vs_cache, tuple(new_lses), tuple(new_msgs))
