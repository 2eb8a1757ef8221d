"""GPU parity of the KV-cache decode kernel (one query row per head against a
long cache) against the numpy oracle, at the head sizes and GQA ratios of the
decode configuration (d 64 / 128, heads / kv_heads up to 4)."""
import numpy as np
import pytest
import torch

from oracle import poly_oracle as O

pytestmark = pytest.mark.gpu
ATOL, RTOL = 2e-2, 1e-2


def rnd(shape, seed):
    return np.random.default_rng(seed).standard_normal(shape).astype(np.float32)


def dev(a, dtype):
    return torch.as_tensor(np.ascontiguousarray(a)).to("cuda", dtype)


def host(t):
    return t.detach().float().cpu().numpy()


@pytest.mark.parametrize("d", [64, 128])
@pytest.mark.parametrize("h,g", [(4, 4), (16, 4), (8, 1)])
@pytest.mark.parametrize("L", [1, 37, 2049])
@pytest.mark.parametrize("extras", ["none", "bias", "bias+vmul+epi"])
def test_decode_pass(d, h, g, L, extras):
    import poly_attention_b200 as P
    dt = torch.bfloat16
    b = 2
    q = host(dev(rnd((b, h, 1, d), 1), dt))
    k, v, vm = (host(dev(rnd((b, g, L, d), s), dt)) for s in (2, 3, 4))
    em = host(dev(rnd((b, h, 1, d), 5), dt))
    bias = rnd((b, g, L), 6)
    kw = {}
    vv = v
    if "bias" in extras:
        kw["bias"] = dev(bias, torch.float32)
    if "vmul" in extras:
        kw["v_mul"] = dev(vm, dt)
        vv = host(dev(v * vm, dt))          # the kernel rounds v * v_mul to bf16, as the reference's product does
    qt, kt, vt = dev(q, dt), dev(k, dt), dev(v, dt)
    assert P.kernel_names(qt, kt, vt)[0] == "decode"
    if "epi" in extras:
        out, lse, eo = P.pass_fwd(qt, kt, vt, epi_mul=dev(em, dt), **kw)
    else:
        out, lse = P.pass_fwd(qt, kt, vt, **kw)
    r = h // g
    eo_, el = O.pass_fwd(q, np.repeat(k, r, 1), np.repeat(vv, r, 1),
                         bias=np.repeat(bias, r, 1) if "bias" in extras else None)
    np.testing.assert_allclose(host(out), eo_, atol=ATOL, rtol=RTOL)
    np.testing.assert_allclose(host(lse), el, atol=ATOL, rtol=RTOL)
    if "epi" in extras:
        np.testing.assert_allclose(host(eo), em * host(out), atol=ATOL, rtol=RTOL)


@pytest.mark.parametrize("order,d", [(2, 64), (3, 128)])
def test_npoly_kv_cache_decode_matches_parallel(order, d):
    """Stepwise KV-cache decoding equals the parallel causal forward
    (the reference's own relation, tests/test_poly_attention.py:139-158), in
    bf16 through the decode kernel, and both match the oracle module."""
    import poly_attention_b200 as P
    torch.manual_seed(3)
    heads, kvh, n = 4, 2, 24
    m = P.NPolyAttention(dim=heads * d, order=order, heads=heads, kv_heads=kvh, dim_head=d, causal=True)
    params = {k: v.detach().float().numpy() for k, v in m.state_dict().items()}
    m = m.cuda().to(torch.bfloat16)
    x = torch.randn(2, n, heads * d)
    xb = x.cuda().to(torch.bfloat16)
    with torch.no_grad():
        par = m(xb)
        cache, outs = None, []
        for i in range(n):
            o, cache = m(xb[:, i:i + 1], cache=cache, return_cache=True)
            outs.append(o)
        step = torch.cat(outs, -2)
    xq = host(xb)
    ref = O.npoly_module_fwd({k: host(dev(v, torch.bfloat16)) for k, v in params.items()}, xq, order=order,
                             heads=heads, kv_heads=kvh, causal=True)
    scale = float(np.abs(ref).max())
    np.testing.assert_allclose(host(par), ref, atol=ATOL * scale, rtol=RTOL)
    np.testing.assert_allclose(host(step), ref, atol=ATOL * scale, rtol=RTOL)


@pytest.mark.parametrize("order,d,h,g", [(2, 64, 4, 2), (3, 128, 16, 4), (4, 64, 4, 4)])
def test_chain_decoder_matches_parallel_oracle(order, d, h, g):
    """Preallocated-cache decoding, one row per step, equals the oracle's
    parallel causal chain (n_poly_attention.py:233-313)."""
    from poly_attention_b200.decode import ChainDecoder
    dt = torch.bfloat16
    b, n = 2, 40
    q1 = host(dev(rnd((b, h, n, d), 1), dt))
    qs = [host(dev(rnd((b, g, n, d), 10 + t), dt)) for t in range(order)]
    vs = [host(dev(rnd((b, g, n, d), 20 + t), dt)) for t in range(order - 1)]
    dec = ChainDecoder(batch=b, order=order, heads=h, kv_heads=g, dim_head=d, capacity=64, dtype=dt)
    outs = []
    for i in range(n):
        dec.append_kv([dev(x[:, :, i:i + 1], dt) for x in qs], [dev(x[:, :, i:i + 1], dt) for x in vs])
        outs.append(host(dec.step(dev(q1[:, :, i:i + 1], dt))))
    got = np.concatenate(outs, axis=2)
    r = h // g
    rep = lambda x: np.repeat(x, r, 1)  # noqa: E731
    ref, _, _ = O.npoly_chain_fwd([q1] + [rep(x) for x in qs[:-1]], [rep(x) for x in qs], [rep(x) for x in vs],
                                  causal=True)
    np.testing.assert_allclose(got, ref, atol=ATOL, rtol=RTOL)
