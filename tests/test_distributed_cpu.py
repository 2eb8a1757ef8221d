"""Key-split long-context order-2 forward: the sharding, the all-gathers of
q2 / q3 / v3 and of pass 1's (msg, lse), and the per-rank passes, run as gloo
ranks on CPU with
the attention passes supplied by the oracle (the CUDA kernels are checked by
the GPU tests). Must equal the oracle's full-sequence causal forward."""
import math
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import poly_oracle as O


def cpu_pass(q, k, v, *, causal=False, softclamp=None, bias=None, causal_offset=0):
    if causal_offset:
        # queries are rows [off, off + nq) of the key sequence: pad them in front
        # so the oracle's top-left causal mask applies, then drop the padding
        pad = torch.zeros(*q.shape[:2], causal_offset, q.shape[-1], dtype=q.dtype)
        out, lse = cpu_pass(torch.cat([pad, q], -2), k, v, causal=causal, softclamp=softclamp, bias=bias)
        return out[..., causal_offset:, :], lse[..., causal_offset:]
    out, lse = O.pass_fwd(q.double().numpy(), k.double().numpy(), v.double().numpy(), causal=causal,
                          softclamp_value=softclamp, bias=None if bias is None else bias.double().numpy())
    return torch.from_numpy(out).float(), torch.from_numpy(lse).float()


def cpu_merge(parts_out, parts_lse):
    m = parts_lse.max(0).values
    w = torch.where(torch.isfinite(parts_lse), torch.exp(parts_lse - m), torch.zeros_like(parts_lse))
    s = w.sum(0)
    out = (parts_out * w[..., None]).sum(0) / s.clamp_min(1e-30)[..., None]
    lse = torch.where(s > 0, m + torch.log(s), torch.full_like(s, -math.inf))
    return out, lse


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, inputs, sc, results):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from poly_attention_b200.distributed import context_parallel_order2_fwd, zigzag_shard
    q1, q2, q3, v3 = (zigzag_shard(t, rank, world) for t in inputs)
    out = context_parallel_order2_fwd(q1, q2, q3, v3, softclamp_value=sc, pass_fn=cpu_pass, merge_fn=cpu_merge)
    results[rank] = out
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [1, 2, 4])
@pytest.mark.parametrize("sc", [None, 20.0])
def test_context_parallel_matches_full_forward(world, sc):
    from poly_attention_b200.distributed import zigzag_unshard
    b, h, d, C = 1, 2, 16, 6 if world != 2 else 128   # C = 128: the one-launch offset path at 2 ranks
    n = 2 * world * C
    g = torch.Generator().manual_seed(world + (sc is not None))
    inputs = [torch.randn(b, h, n, d, generator=g) for _ in range(4)]
    results = mp.Manager().dict()
    mp.spawn(_worker, args=(world, _free_port(), inputs, sc, results), nprocs=world, join=True)
    out = zigzag_unshard([results[r] for r in range(world)], world)
    q1, q2, q3, v3 = (t.numpy().astype(np.float64) for t in inputs)
    ref, _, _ = O.order2_fwd(q1, q2, q2, q3, v3, softclamp_value=sc, causal=True)
    np.testing.assert_allclose(out.numpy(), ref, atol=1e-5, rtol=1e-5)


def test_zigzag_roundtrip():
    from poly_attention_b200.distributed import zigzag_shard, zigzag_unshard
    x = torch.arange(2 * 3 * 4).reshape(1, 1, 24, 1).float()
    parts = [zigzag_shard(x, r, 3) for r in range(3)]
    assert parts[0][0, 0, :, 0].tolist() == [0, 1, 2, 3, 20, 21, 22, 23]
    assert torch.equal(zigzag_unshard(parts, 3), x)
