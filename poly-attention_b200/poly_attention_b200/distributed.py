"""Long-context order-2 poly attention with the keys split across GPUs.

One process per GPU (torch.distributed, NCCL). The sequence of n rows is cut
into 2P chunks of C = n / (2P) rows; rank r owns chunks r and 2P-1-r
("zig-zag", which balances the causal work). Each rank holds the rows of its
chunks of q1, q2, q3, v3 (``[b, h, 2C, d]``, chunk r first) and produces the
output rows of those chunks.

Forward (causal, reference semantics of poly_attention/poly_attention.py:48-116):

1. all-gather q3, v3 (pass 1's keys / values) and q2 (pass 2's keys), stacked
   into one message, then reassembled in natural row order.
2. pass 1 for the own rows of q2 against every key up to the row: one causal
   launch with the key index offset by the chunk start (or, for chunks not a
   multiple of 128 rows, the earlier chunks unmasked plus the diagonal chunk
   causal, merged by log-sum-exp) -> (msg, lse23) of the own rows, complete
   (pass-1 rows are exactly pass-2 keys).
3. all-gather msg and lse23: every rank now holds pass 2's keys (q2), values
   (msg) and key bias (lse23) for the whole sequence.
4. pass 2 for the own rows of q1, the same way: complete output rows, no
   partial results leave the rank.

Per rank this receives 4 (n x d) 16-bit tensors and one n-row fp32 vector
(times (P - 1) / P) and never sends q1; the compute is 2 x n x 2C key-query
pairs per pass (balanced by the zig-zag). The attention passes are the CUDA
kernels (``ops.pass_fwd`` / ``ops.lse_merge``); ``pass_fn`` / ``merge_fn`` can
be replaced, which the CPU tests use to check the collective logic with the
gloo backend.
"""
from __future__ import annotations

import math

import torch
import torch.distributed as dist


def zigzag_chunks(rank: int, world: int):
    """The two chunk indices (of 2 * world) rank `rank` owns."""
    return rank, 2 * world - 1 - rank


def zigzag_shard(x: torch.Tensor, rank: int, world: int, dim: int = -2) -> torch.Tensor:
    """Rows of `x` (full sequence on `dim`) that rank `rank` owns, chunk r first."""
    c = x.shape[dim] // (2 * world)
    a, b = zigzag_chunks(rank, world)
    return torch.cat([x.narrow(dim, a * c, c), x.narrow(dim, b * c, c)], dim=dim)


def zigzag_unshard(parts, world: int, dim: int = -2) -> torch.Tensor:
    """Inverse of zigzag_shard: list of per-rank shards -> full sequence."""
    c = parts[0].shape[dim] // 2
    chunks = [None] * (2 * world)
    for r, p in enumerate(parts):
        a, b = zigzag_chunks(r, world)
        chunks[a] = p.narrow(dim, 0, c)
        chunks[b] = p.narrow(dim, c, c)
    return torch.cat(chunks, dim=dim)


def _gather_start(x_loc, world, group):
    """Start an all-gather of this rank's zig-zag shard into one flat
    [world, ...] buffer; returns a handle for _gather_finish (no collective
    at world size 1)."""
    x_loc = x_loc.contiguous()
    if world == 1:
        return x_loc, None
    flat = x_loc.new_empty((world * x_loc.shape[0], *x_loc.shape[1:]))   # ranks along dim 0
    work = dist.all_gather_into_tensor(flat, x_loc, group=group, async_op=True)
    return flat.view(world, *x_loc.shape), work


def _gather_finish(handle, world, dim=-2):
    """Wait for the gather (stream-ordered with NCCL) and reassemble the
    natural row order along `dim`."""
    flat, work = handle
    if work is not None:
        work.wait()
    return flat if world == 1 else zigzag_unshard(list(flat.unbind(0)), world, dim=dim)


def _default_ops():
    from .ops import lse_merge, pass_fwd
    return pass_fwd, lse_merge


def context_parallel_order2_fwd(q1_loc, q2_loc, q3_loc, v3_loc, *, group=None, softclamp_value=None,
                                pass_fn=None, merge_fn=None):
    """Causal order-2 poly attention forward over a key-split sequence.

    All inputs are this rank's zig-zag shard ``[b, h, 2C, d]``. Returns this
    rank's shard of the output (same layout, input dtype).
    """
    if pass_fn is None or merge_fn is None:
        pf, mf = _default_ops()
        pass_fn = pass_fn or pf
        merge_fn = merge_fn or mf
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    rank = dist.get_rank(group) if dist.is_initialized() else 0
    C = q1_loc.shape[-2] // 2
    own = zigzag_chunks(rank, world)
    sc = softclamp_value

    # q3, v3 and q2 travel in one gather (one large message moves faster than
    # three); stacked along a new leading axis, split again after
    h_kv = _gather_start(torch.stack([q3_loc, v3_loc, q2_loc]), world, group) if world > 1 else None
    rows = lambda x, k, dim=-2: x.narrow(dim, k * C, C)   # noqa: E731  (own chunk k of a local shard)

    def diag(q_rows, k, v, bias):
        """Rows of an own chunk against the same chunk's keys (causal; both
        index ranges start at the chunk start, so the top-left rule is exact)."""
        return pass_fn(q_rows, k, v, causal=True, softclamp=sc, bias=bias)

    def prefix(q_rows, c, part, k, v, bias):
        """Add the keys of the chunks before c (no mask) to a diagonal result."""
        if c == 0:
            return part
        o_p, l_p = pass_fn(q_rows, k[:, :, :c * C], v[:, :, :c * C], causal=False, softclamp=sc,
                           bias=None if bias is None else bias[:, :, :c * C])
        return merge_fn(torch.stack([o_p, part[0]]), torch.stack([l_p, part[1]]))

    def whole(q_rows, c, k, v, bias):
        """Rows of chunk c against keys [0, (c + 1) C) in one causal launch with
        the key index offset by c * C (C a multiple of the 128-key tile)."""
        if c == 0:
            return diag(q_rows, k[:, :, :C], v[:, :, :C], None if bias is None else bias[:, :, :C])
        return pass_fn(q_rows, k[:, :, :(c + 1) * C], v[:, :, :(c + 1) * C], causal=True, softclamp=sc,
                       bias=None if bias is None else bias[:, :, :(c + 1) * C], causal_offset=c * C)

    # one offset launch per own chunk (or, for chunks not a multiple of the
    # 128-key tile, the diagonal block and the earlier chunks merged). Running
    # the diagonal blocks on local data while the gathers are in flight was
    # measured slower: the pass kernels hold every SM, so NCCL's gather kernels
    # wait for them instead of overlapping.
    def attend(q_rows, c, k, v, bias):
        if C % 128 == 0:
            return whole(q_rows, c, k, v, bias)
        sl = slice(c * C, (c + 1) * C)
        part = diag(q_rows, k[:, :, sl], v[:, :, sl], None if bias is None else bias[:, :, sl])
        return prefix(q_rows, c, part, k, v, bias)

    # pass 1 for the own rows of q2 (poly_attention/poly_attention.py:63-82)
    q3, v3, q2 = _gather_finish(h_kv, world).unbind(0) if world > 1 else (q3_loc, v3_loc, q2_loc)
    res = [attend(rows(q2_loc, k), c, q3, v3, None) for k, c in enumerate(own)]
    del q3, v3
    h_msg = _gather_start(torch.cat([r[0] for r in res], dim=-2), world, group)
    h_lse = _gather_start(torch.cat([r[1] for r in res], dim=-1), world, group)
    del res

    # pass 2 for the own rows of q1, lse23 as key bias (:91-114)
    msg = _gather_finish(h_msg, world)
    lse23 = _gather_finish(h_lse, world, dim=-1)
    outs = [attend(rows(q1_loc, k), c, q2, msg, lse23)[0] for k, c in enumerate(own)]
    return torch.cat(outs, dim=-2).to(q1_loc.dtype)
