"""Long-context order-2 poly attention with the keys split across GPUs.

One process per GPU (torch.distributed, NCCL). The sequence of n rows is cut
into 2P chunks of C = n / (2P) rows; rank r owns chunks r and 2P-1-r
("zig-zag", which balances the causal work). Each rank holds the rows of its
chunks of q1, q2, q3, v3 (``[b, h, 2C, d]``, chunk r first).

Forward (causal, reference semantics of poly_attention/poly_attention.py:48-116):

1. all-gather q1, q3, v3 (q2 stays local: pass 1's queries and pass 2's keys
   are the rank's own rows).
2. pass 1 for the own rows: keys of earlier chunks without mask plus the
   diagonal chunk with the causal mask, merged by log-sum-exp -> (msg, lse23)
   of the own rows, complete: pass-1 rows are exactly pass-2 keys.
3. pass 2, key split: for each own key chunk c, the queries of chunk c
   (causal) and of every later chunk (no mask) attend keys c with lse23 as key
   bias, as one causal call -> partial (out, lse) for every query row; the two
   own chunks are merged locally (poly_lse_merge).
4. the one exchange: all-reduce(max) of the partial lse per row, each rank
   rescales its partial by exp(lse - max), then reduce-scatter(sum) of
   [acc | l] (fp32) delivers every row's totals to its owner, which divides.

The attention passes are the CUDA kernels (``ops.pass_fwd`` / ``ops.lse_merge``);
``pass_fn`` / ``merge_fn`` can be replaced, which the CPU tests use to check
the collective logic with the gloo backend.
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


def _gather_full(x_loc, world, group):
    """all-gather zig-zag shards and reassemble the natural row order."""
    if world == 1:
        return zigzag_unshard([x_loc], 1)
    parts = [torch.empty_like(x_loc) for _ in range(world)]
    dist.all_gather(parts, x_loc.contiguous(), group=group)
    return zigzag_unshard(parts, world)


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
    b, h, n2, d = q1_loc.shape
    C = n2 // 2
    n = C * 2 * world
    ca, cb = zigzag_chunks(rank, world)
    own = (ca, cb)

    q1 = _gather_full(q1_loc, world, group)
    q3 = _gather_full(q3_loc, world, group)
    v3 = _gather_full(v3_loc, world, group)
    rows = lambda x, c: x[:, :, c * C:(c + 1) * C]  # noqa: E731

    # 2. pass 1 for the own rows (keys <= row): earlier chunks unmasked + diagonal causal
    msgs, lses = [], []
    for k, c in enumerate(own):
        q2c = q2_loc[:, :, k * C:(k + 1) * C]
        o_d, l_d = pass_fn(q2c, rows(q3, c), rows(v3, c), causal=True, softclamp=softclamp_value)
        if c > 0:
            o_p, l_p = pass_fn(q2c, q3[:, :, :c * C], v3[:, :, :c * C], causal=False, softclamp=softclamp_value)
            o_d, l_d = merge_fn(torch.stack([o_p, o_d]), torch.stack([l_p, l_d]))
        msgs.append(o_d)
        lses.append(l_d)

    # 3. pass 2 partials for every query row from the own key chunks. Queries
    # from chunk c on against keys of chunk c is one causal call: with both
    # index ranges starting at c * C, the top-left causal rule masks exactly
    # the diagonal block and leaves the later rows unmasked.
    part_out = torch.empty(2, b, h, n, d, device=q1.device, dtype=q1.dtype)
    part_lse = torch.empty(2, b, h, n, device=q1.device, dtype=torch.float32)
    for k, c in enumerate(own):
        q2c = q2_loc[:, :, k * C:(k + 1) * C]
        o, l = pass_fn(q1[:, :, c * C:], q2c, msgs[k], causal=True, softclamp=softclamp_value, bias=lses[k])
        part_out[k, :, :, c * C:] = o
        part_lse[k, :, :, c * C:] = l
        part_out[k, :, :, :c * C] = 0        # rows before chunk c see none of its keys
        part_lse[k, :, :, :c * C] = -math.inf
    out_p, lse_p = merge_fn(part_out, part_lse)

    # 4. exchange: max of lse, then sum of rescaled [acc | l] to the row owners
    m = lse_p.clone()
    if world > 1:
        dist.all_reduce(m, op=dist.ReduceOp.MAX, group=group)
    w = torch.where(torch.isfinite(lse_p), torch.exp(lse_p - m), torch.zeros_like(lse_p))
    buf = torch.cat([out_p.float() * w[..., None], w[..., None]], dim=-1)           # [b, h, n, d + 1]
    # zig-zag order so that reduce-scatter's contiguous blocks are the owners' rows
    blocks = [zigzag_shard(buf, r, world) for r in range(world)]
    if world > 1:
        mine = torch.empty_like(blocks[0])
        dist.reduce_scatter(mine, [x.contiguous() for x in blocks], op=dist.ReduceOp.SUM, group=group)
    else:
        mine = blocks[0]
    acc, l = mine[..., :d], mine[..., d:]
    out = torch.where(l > 0, acc / l.clamp_min(1e-30), torch.zeros_like(acc))
    return out.to(q1_loc.dtype)
