"""Module-level KV cache: the tuples PolyAttention / NPolyAttention return are
views of capacity-doubling buffers that the next step appends to in place
(instead of the reference's per-step torch.cat, poly_attention.py:283-287,
n_poly_attention.py:206-207). Checked: stepwise decoding equals the parallel
forward (the reference's own invariant, tests/test_poly_attention.py:103-119),
steps write in place, growth past the capacity, and a stale / foreign cache
tuple (a branch of the sequence) gives the same result as a fresh one.
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _mods(dtype):
    import poly_attention_b200 as P
    torch.manual_seed(0)
    m2 = P.PolyAttention(dim=128, heads=8, kv_heads=2, dim_head=64, causal=True).cuda().to(dtype)
    m3 = P.NPolyAttention(dim=128, order=3, heads=8, kv_heads=2, dim_head=64, causal=True,
                          softclamp_value=20.0).cuda().to(dtype)
    return m2, m3


def _tol(dtype):
    return dict(atol=1e-4, rtol=1e-4) if dtype == torch.float32 else dict(atol=2e-2, rtol=1e-2)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_stepwise_equals_parallel_and_appends_in_place(dtype):
    for m in _mods(dtype):
        x = torch.randn(2, 150, 128, device="cuda", dtype=dtype)
        with torch.no_grad():
            full = m(x)
            n0 = 10
            out, cache = m(x[:, :n0], return_cache=True)      # prefill: capacity max(2 n, n + 64) = 74
            outs = [out]
            ptrs = None
            grew = 0
            for i in range(n0, x.shape[1]):
                out, cache = m(x[:, i:i + 1], cache=cache, return_cache=True)
                outs.append(out)
                flat = [t for part in cache for t in (part if isinstance(part, tuple) else (part,))]
                now = [t.data_ptr() for t in flat]
                if ptrs is not None and now != ptrs:
                    grew += 1
                ptrs = now
                assert all(t.shape[2] == i + 1 for t in flat)
        np.testing.assert_allclose(torch.cat(outs, 1).float().cpu().numpy(), full.float().cpu().numpy(),
                                   **_tol(dtype))
        assert grew == 2, grew          # capacity 74 -> 148 -> 296 rows over 140 steps past a 10-row prefill


def test_branching_and_foreign_cache():
    dtype = torch.bfloat16
    m2, m3 = _mods(dtype)
    for m in (m2, m3):
        x = torch.randn(1, 40, 128, device="cuda", dtype=dtype)
        with torch.no_grad():
            _, c20 = m(x[:, :20], return_cache=True)
            _, c21 = m(x[:, 20:21], cache=c20, return_cache=True)
            a, _ = m(x[:, 21:22], cache=c21, return_cache=True)
            # branch: step from the older cache with another token, then from c21 again
            b_, _ = m(x[:, 30:31], cache=c20, return_cache=True)
            a2, _ = m(x[:, 21:22], cache=c21, return_cache=True)
            ref_b = m(torch.cat([x[:, :20], x[:, 30:31]], 1))[:, -1:]
            ref_a = m(x[:, :22])[:, -1:]
        for got, want in ((a, ref_a), (a2, ref_a), (b_, ref_b)):
            np.testing.assert_allclose(got.float().cpu().numpy(), want.float().cpu().numpy(), atol=2e-2, rtol=1e-2)
