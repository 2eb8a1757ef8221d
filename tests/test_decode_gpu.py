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
@pytest.mark.parametrize("h,g", [(4, 4), (16, 4), (8, 4), (8, 1)])
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


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("d,h,g,L", [(64, 8, 4, 300), (128, 16, 2, 20000), (128, 4, 4, 65), (64, 2, 1, 4096)])
def test_decode_pass_softclamp_dead_keys(dt, d, h, g, L):
    """Softclamp, fp16, GQA ratios 2 and 8, long caches (the largest split
    count) and dead keys (bias <= -FLT_MAX / 2, the previous level's lse of a
    fully masked row) together."""
    import poly_attention_b200 as P
    b = 2
    q = host(dev(rnd((b, h, 1, d), 11), dt))
    k, v, vm = (host(dev(rnd((b, g, L, d), s), dt)) for s in (12, 13, 14))
    bias = rnd((b, g, L), 15)
    bias[:, :, ::7] = -np.finfo(np.float32).max
    vv = host(dev(v * vm, dt))
    qt, kt, vt = dev(q, dt), dev(k, dt), dev(v, dt)
    assert P.kernel_names(qt, kt, vt)[0] == "decode"
    out, lse = P.pass_fwd(qt, kt, vt, softclamp=10.0, bias=dev(bias, torch.float32), v_mul=dev(vm, dt))
    r = h // g
    eo_, el = O.pass_fwd(q, np.repeat(k, r, 1), np.repeat(vv, r, 1), softclamp_value=10.0,
                         bias=np.repeat(bias, r, 1))
    np.testing.assert_allclose(host(out), eo_, atol=ATOL, rtol=RTOL)
    np.testing.assert_allclose(host(lse), el, atol=ATOL, rtol=RTOL)


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


@pytest.mark.parametrize("order,d,h,g,L0", [(3, 128, 16, 4, 3000), (4, 64, 8, 2, 700)])
def test_decode_chain_equals_level_by_level(order, d, h, g, L0):
    """One poly_decode_chain call per step (levels launched as programmatic
    dependents, each streaming its cache before waiting for the previous
    level) gives bit-identical results to the same kernels launched level by
    level with full stream serialisation, over many steps of long caches."""
    from poly_attention_b200.decode import ChainDecoder
    dt = torch.bfloat16
    b, steps = 4, 24
    gen = torch.Generator(device="cuda").manual_seed(3)
    decs = [ChainDecoder(batch=b, order=order, heads=h, kv_heads=g, dim_head=d, capacity=L0 + steps + 8, dtype=dt)
            for _ in range(2)]
    for bufs in zip(*[dd.qs + dd.vs + dd.msgs + dd.lses for dd in decs]):
        bufs[0][:, :, :L0].normal_(generator=gen)
        bufs[1].copy_(bufs[0])
    for dd in decs:
        dd.length = L0
    decs[1]._chain = False
    for i in range(steps):
        qn = [torch.randn(b, g, 1, d, device="cuda", dtype=dt, generator=gen) for _ in range(order)]
        vn = [torch.randn(b, g, 1, d, device="cuda", dtype=dt, generator=gen) for _ in range(order - 1)]
        q1 = torch.randn(b, h, 1, d, device="cuda", dtype=dt, generator=gen)
        outs = []
        for dd in decs:
            dd.append_kv(qn, vn)
            outs.append(dd.step(q1).clone())
        assert torch.equal(outs[0], outs[1]), f"step {i}"
    assert decs[0]._chain is True
    for m0, m1 in zip(decs[0].msgs + decs[0].lses, decs[1].msgs + decs[1].lses):
        assert torch.equal(m0[:, :, :L0 + steps], m1[:, :, :L0 + steps])


def test_copy_rows_matches_slice_assignment():
    """poly_copy_rows (every cache append of a step in one launch) writes the
    same bytes as slice assignment, for strided sources and destinations of
    several row sizes, and leaves every other row untouched."""
    import ctypes
    from poly_attention_b200 import _lib
    gen = torch.Generator(device="cuda").manual_seed(9)
    dsts, srcs, refs = [], [], []
    cps = (_lib.PolyRowCopy * 5)()
    for i, (b, g, d, dt) in enumerate([(3, 4, 64, torch.bfloat16), (2, 1, 128, torch.float16), (5, 2, 8, torch.float32),
                                       (1, 8, 128, torch.bfloat16), (4, 3, 96, torch.bfloat16)]):
        cache = torch.randn(b, g, 50, d, device="cuda", generator=gen).to(dt)
        src = torch.randn(b, 2 * g, 1, d, device="cuda", generator=gen).to(dt)[:, ::2]   # strided heads
        row = 7 * i + 3
        ref = cache.clone()
        ref[:, :, row:row + 1] = src
        e = cache.element_size()
        c = cps[i]
        c.src, c.dst = src.data_ptr(), cache.data_ptr() + row * cache.stride(2) * e
        c.outer, c.inner, c.row_bytes = b, g, d * e
        c.src_stride[0], c.src_stride[1] = src.stride(0) * e, src.stride(1) * e
        c.dst_stride[0], c.dst_stride[1] = cache.stride(0) * e, cache.stride(1) * e
        dsts.append(cache)
        refs.append(ref)
        srcs.append(src)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    assert _lib.lib.poly_copy_rows(cps, 5, stream) == _lib.POLY_OK
    torch.cuda.synchronize()
    for got, ref in zip(dsts, refs):
        assert torch.equal(got, ref)


@pytest.mark.parametrize("vmul", [False, True])
def test_decode_fully_dead_keys(vmul):
    """Every cached key dead for one sequence (its previous-level rows were
    fully masked): the reference's uniform average of the values, lse = -FLT_MAX."""
    import poly_attention_b200 as P
    dt = torch.bfloat16
    b, h, g, L, d = 2, 8, 2, 300, 128
    q = host(dev(rnd((b, h, 1, d), 21), dt))
    k, v, vm = (host(dev(rnd((b, g, L, d), s), dt)) for s in (22, 23, 24))
    bias = rnd((b, g, L), 25)
    bias[0] = -np.finfo(np.float32).max
    kw = {"bias": dev(bias, torch.float32)}
    vv = v
    if vmul:
        kw["v_mul"] = dev(vm, dt)
        vv = host(dev(v * vm, dt))
    qt, kt, vt = dev(q, dt), dev(k, dt), dev(v, dt)
    assert P.kernel_names(qt, kt, vt)[0] == "decode"
    out, lse = P.pass_fwd(qt, kt, vt, **kw)
    r = h // g
    eo_, el = O.pass_fwd(q, np.repeat(k, r, 1), np.repeat(vv, r, 1), bias=np.repeat(bias, r, 1))
    np.testing.assert_allclose(host(out), eo_, atol=ATOL, rtol=RTOL)
    np.testing.assert_allclose(host(lse), el, atol=ATOL, rtol=RTOL)


@pytest.mark.parametrize("extras", ["none", "bias+vmul+epi", "dead"])
@pytest.mark.parametrize("b,h,g,L,d", [(1, 8, 2, 20000, 128), (1, 4, 4, 12000, 64), (2, 16, 2, 12000, 128)])
def test_decode_global_split(b, h, g, L, d, extras):
    """Few (batch, kv head) groups and long caches take the global-split mode
    (up to 64 splits per group, CTA records merged by a combine kernel)."""
    import poly_attention_b200 as P
    dt = torch.bfloat16
    q = host(dev(rnd((b, h, 1, d), 31), dt))
    k, v, vm = (host(dev(rnd((b, g, L, d), s), dt)) for s in (32, 33, 34))
    em = host(dev(rnd((b, h, 1, d), 35), dt))
    bias = rnd((b, g, L), 36)
    kw, vv, obias = {}, v, None
    if extras == "dead":
        bias[0] = -np.finfo(np.float32).max
    if extras != "none":
        kw["bias"], obias = dev(bias, torch.float32), np.repeat(bias, h // g, 1)
    if "vmul" in extras:
        kw["v_mul"] = dev(vm, dt)
        vv = host(dev(v * vm, dt))
    qt, kt, vt = dev(q, dt), dev(k, dt), dev(v, dt)
    assert P.kernel_names(qt, kt, vt)[0] == "decode"
    from poly_attention_b200 import _lib
    n0 = _lib.launch_count()
    if "epi" in extras:
        out, lse, eo = P.pass_fwd(qt, kt, vt, epi_mul=dev(em, dt), **kw)
    else:
        out, lse = P.pass_fwd(qt, kt, vt, **kw)
    assert _lib.launch_count() - n0 == 2   # split kernel + combine kernel
    r = h // g
    eo_, el = O.pass_fwd(q, np.repeat(k, r, 1), np.repeat(vv, r, 1), bias=obias)
    np.testing.assert_allclose(host(out), eo_, atol=ATOL, rtol=RTOL)
    np.testing.assert_allclose(host(lse), el, atol=ATOL, rtol=RTOL)
    if "epi" in extras:
        np.testing.assert_allclose(host(eo), em * host(out), atol=ATOL, rtol=RTOL)


def test_chain_decoder_single_sequence_long_cache():
    """Batch 1 through ChainDecoder (global-split levels inside poly_decode_chain)
    equals the level-by-level launches."""
    from poly_attention_b200.decode import ChainDecoder
    dt = torch.bfloat16
    b, order, h, g, d, L0, steps = 1, 3, 16, 4, 128, 12000, 6
    gen = torch.Generator(device="cuda").manual_seed(8)
    decs = [ChainDecoder(batch=b, order=order, heads=h, kv_heads=g, dim_head=d, capacity=L0 + steps + 8, dtype=dt)
            for _ in range(2)]
    for bufs in zip(*[dd.qs + dd.vs + dd.msgs + dd.lses for dd in decs]):
        bufs[0][:, :, :L0].normal_(generator=gen)
        bufs[1].copy_(bufs[0])
    for dd in decs:
        dd.length = L0
    decs[1]._chain = False
    for _ in range(steps):
        qn = [torch.randn(b, g, 1, d, device="cuda", dtype=dt, generator=gen) for _ in range(order)]
        vn = [torch.randn(b, g, 1, d, device="cuda", dtype=dt, generator=gen) for _ in range(order - 1)]
        q1 = torch.randn(b, h, 1, d, device="cuda", dtype=dt, generator=gen)
        outs = []
        for dd in decs:
            dd.append_kv(qn, vn)
            outs.append(dd.step(q1).clone())
        assert torch.equal(outs[0], outs[1])
    assert decs[0]._chain is True
