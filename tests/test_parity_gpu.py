"""GPU parity: the CUDA library against the numpy oracle (itself pinned to the
reference by tests/test_oracle_golden.py) and against the golden vectors.

Tolerances (stated by the build's target): fp32 paths within 1e-4 max-abs;
bf16 kernels against the fp32 oracle within max-abs 2e-2 / rel 1e-2.
"""
import numpy as np
import pytest
import torch

from oracle import poly_oracle as O

pytestmark = pytest.mark.gpu

FP32_ATOL = 1e-4
BF16_ATOL, BF16_RTOL = 2e-2, 1e-2


def dev(a, dtype=torch.float32):
    return torch.as_tensor(np.ascontiguousarray(a)).to("cuda", dtype)


def host(t):
    return t.detach().float().cpu().numpy()


def assert_close(got, want, dtype, what=""):
    got = host(got) if torch.is_tensor(got) else got
    if dtype == torch.float32:
        np.testing.assert_allclose(got, want, atol=FP32_ATOL, rtol=0, err_msg=what)
    else:
        np.testing.assert_allclose(got, want, atol=BF16_ATOL, rtol=BF16_RTOL, err_msg=what)


def rnd(shape, seed):
    return np.random.default_rng(seed).standard_normal(shape).astype(np.float32)


def quant(a, dtype):
    """Round to the kernel's input dtype so the oracle sees the same inputs."""
    return host(dev(a, dtype))


# ---------------------------------------------------------------- single pass

@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("nq,nk,d", [(31, 31, 64), (128, 128, 64), (200, 200, 128), (17, 40, 32)])
def test_pass_fwd(dtype, causal, nq, nk, d):
    import poly_attention_b200 as P
    b, h, g = 2, 4, 2
    q, k, v = (quant(rnd(s, i), dtype) for i, s in enumerate([(b, h, nq, d), (b, g, nk, d), (b, g, nk, d)]))
    bias = rnd((b, g, nk), 7)
    out, lse = P.pass_fwd(dev(q, dtype), dev(k, dtype), dev(v, dtype), causal=causal, bias=dev(bias))
    r = h // g
    eo, el = O.pass_fwd(q, np.repeat(k, r, 1), np.repeat(v, r, 1), causal=causal, bias=np.repeat(bias, r, 1))
    assert_close(out, eo, dtype, "out")
    assert_close(lse, el, dtype, "lse")


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_pass_fwd_masks_softclamp_epilogue(dtype):
    import poly_attention_b200 as P
    b, h, n, d = 2, 2, 45, 64
    q, k, v, em = (quant(rnd((b, h, n, d), i + 10), dtype) for i in range(4))
    km = np.ones((b, n), bool); km[0, 30:] = False; km[1, 0] = False
    qm = np.ones((b, n), bool); qm[1, 3] = False
    out, lse, eo_gpu = P.pass_fwd(dev(q, dtype), dev(k, dtype), dev(v, dtype), causal=True, softclamp=20.0,
                                  key_mask=torch.as_tensor(km).cuda(), query_mask=torch.as_tensor(qm).cuda(),
                                  epi_mul=dev(em, dtype))
    eo, el = O.pass_fwd(q, k, v, causal=True, softclamp_value=20.0, key_mask=km, query_mask=qm)
    assert_close(out, eo, dtype, "out")
    # fully excluded rows give lse = -finfo.max in the reference; compare finite rows
    fin = el > -1e30
    assert_close(host(lse)[fin], el[fin], dtype, "lse")
    assert np.all(host(lse)[~fin] < -1e30)
    assert_close(eo_gpu, em * host(out), dtype, "epilogue")


def test_pass_fwd_v_mul():
    import poly_attention_b200 as P
    b, h, n, d = 1, 2, 33, 64
    q, k, v, vm = (rnd((b, h, n, d), i + 20) for i in range(4))
    out, lse = P.pass_fwd(dev(q), dev(k), dev(v), v_mul=dev(vm))
    eo, el = O.pass_fwd(q, k, v * vm)
    assert_close(out, eo, torch.float32)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("n", [31, 128])
def test_pass_bwd(dtype, causal, n):
    import poly_attention_b200 as P
    b, h, g, d = 2, 4, 2, 64
    q = quant(rnd((b, h, n, d), 1), dtype)
    k, v = (quant(rnd((b, g, n, d), s), dtype) for s in (2, 3))
    do = quant(rnd((b, h, n, d), 4), dtype)
    bias = rnd((b, g, n), 5)
    dlse = rnd((b, h, n), 6)
    qt, kt, vt = dev(q, dtype), dev(k, dtype), dev(v, dtype)
    out, lse = P.pass_fwd(qt, kt, vt, causal=causal, softclamp=20.0, bias=dev(bias))
    dq, dk, dv, db = P.pass_bwd(qt, kt, vt, out, lse, dev(do, dtype), causal=causal, softclamp=20.0,
                                bias=dev(bias), dlse=dev(dlse), want_dbias=True)
    r = h // g
    edq, edk, edv, edb = O._pass_bwd(q, np.repeat(k, r, 1), np.repeat(v, r, 1), do, scale=d ** -0.5, causal=causal,
                                     softclamp_value=20.0, key_mask=None, query_mask=None,
                                     bias=np.repeat(bias, r, 1), dlse=dlse)
    group = lambda t: t.reshape(b, g, r, *t.shape[2:]).sum(2)  # noqa: E731
    assert_close(dq, edq, dtype, "dq")
    assert_close(dk, group(edk), dtype, "dk")
    assert_close(dv, group(edv), dtype, "dv")
    assert_close(db, group(edb), dtype, "dbias")


# ---------------------------------------------------------------- order 2

@pytest.mark.parametrize("n", [17, 64])
@pytest.mark.parametrize("causal", [0, 1])
@pytest.mark.parametrize("sc", [0, 20])
def test_order2_golden_fwd_bwd(golden, n, causal, sc):
    """reference_poly_attention fwd + autograd grads (golden vectors), fp32."""
    import poly_attention_b200 as P
    gd = golden(f"ref_fn_n{n}_c{causal}_s{sc}")
    t = {k: dev(gd[k]).requires_grad_(True) for k in ("q1", "q2a", "q2b", "q3", "v3")}
    out, lse, msg = P.poly_attention_order2(t["q1"], t["q2b"], t["q3"], t["v3"], q2_pass1=t["q2a"],
                                            softclamp_value=sc or None, causal=bool(causal))
    out.backward(dev(gd["dout"]))
    assert_close(out, gd["out"], torch.float32, "out")
    assert_close(lse, gd["lse23"], torch.float32, "lse23")
    assert_close(msg, gd["msg"], torch.float32, "msg")
    for k in t:
        assert_close(t[k].grad, gd["d" + k], torch.float32, "d" + k)


@pytest.mark.parametrize("causal", [0, 1])
def test_order2_golden_masked(golden, causal):
    import poly_attention_b200 as P
    gd = golden(f"ref_fn_masked_c{causal}")
    t = {k: dev(gd[k]).requires_grad_(True) for k in ("q1", "q2a", "q2b", "q3", "v3")}
    m = {k: torch.as_tensor(gd[k]).cuda() for k in ("mask", "cm1", "cm2")}
    out, lse, msg = P.poly_attention_order2(t["q1"], t["q2b"], t["q3"], t["v3"], q2_pass1=t["q2a"], mask=m["mask"],
                                            context_mask=(m["cm1"], m["cm2"]), causal=bool(causal))
    out.backward(dev(gd["dout"]))
    assert_close(out, gd["out"], torch.float32, "out")
    assert_close(msg, gd["msg"], torch.float32, "msg")
    for k in t:
        assert_close(t[k].grad, gd["d" + k], torch.float32, "d" + k)


@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("seq_len", [31, 32, 127, 128])
@pytest.mark.parametrize("softclamp_value", [None, 20.0])
def test_flash_poly_attention_matches_oracle(causal, seq_len, softclamp_value):
    """Mirror of the reference's flash test (tests/test_poly_attention.py:213-240):
    (2, 4, n, 64), fwd and all four grads; bf16 against the fp32 oracle."""
    import poly_attention_b200 as P
    dtype = torch.bfloat16
    shape = (2, 4, seq_len, 64)
    arrs = [quant(rnd(shape, 42 + i), dtype) for i in range(4)]
    do = quant(rnd(shape, 99), dtype)
    ts = [dev(a, dtype).requires_grad_(True) for a in arrs]
    out = P.flash_poly_attention(*ts, softclamp_value=softclamp_value, is_causal=causal)
    out.backward(dev(do, dtype))
    q1, q2, q3, v3 = arrs
    eo, _, _ = O.order2_fwd(q1, q2, q2, q3, v3, softclamp_value=softclamp_value, causal=causal)
    g = O.order2_bwd(q1, q2, q2, q3, v3, do, softclamp_value=softclamp_value, causal=causal)
    assert_close(out, eo, dtype, "out")
    for i, (t, e) in enumerate(zip(ts, (g[0], g[1] + g[2], g[3], g[4]))):
        assert_close(t.grad, e, dtype, f"grad {i}")


# ---------------------------------------------------------------- order n

@pytest.mark.parametrize("order", [2, 3, 4])
def test_chain_golden_fwd_bwd(golden, order):
    import poly_attention_b200 as P
    gd = golden(f"chain_grad_o{order}")
    qs = [dev(gd[f"q{i}"]).requires_grad_(True) for i in range(order + 1)]
    vs = [dev(gd[f"v{i}"]).requires_grad_(True) for i in range(2, order + 1)]
    out, _, _ = P.poly_attention_chain(qs[:-1], qs[1:], vs, causal=True,
                                       softclamp_value=20.0 if order == 3 else None)
    out.backward(dev(gd["dchain"]))
    assert_close(out, gd["chain_out"], torch.float32, "out")
    for i in range(order + 1):
        assert_close(qs[i].grad, gd[f"dq{i}"], torch.float32, f"dq{i}")
    for i, v in enumerate(vs):
        assert_close(v.grad, gd[f"dv{i + 2}"], torch.float32, f"dv{i + 2}")


# ---------------------------------------------------------------- modules

MOD2 = {
    "base": dict(heads=4),
    "causal_gqa": dict(heads=4, kv_heads=2, causal=True, softclamp_value=20.0),
    "root_gate": dict(heads=4, causal=True, multiply_root_value=True, use_root_value_as_attn_gate=True, attn_gate=True),
    "shared_prenorm": dict(heads=4, kv_heads=1, shared_kv=True, prenorm=True, multiply_root_value=True),
}


def load_module(mod, gd):
    sd = {k[2:]: torch.as_tensor(v) for k, v in gd.items() if k.startswith("p:")}
    mod.load_state_dict(sd)
    return mod.cuda()


@pytest.mark.parametrize("name", sorted(MOD2))
def test_order2_module_golden(golden, name):
    import poly_attention_b200 as P
    gd = golden(f"mod2_{name}")
    m = load_module(P.PolyAttention(dim=64, dim_head=16, **MOD2[name]), gd)
    with torch.no_grad():
        y = m(dev(gd["x"]))
    assert_close(y, gd["y"], torch.float32)


def test_order2_module_context_masks_golden(golden):
    import poly_attention_b200 as P
    gd = golden("mod2_context_masks")
    m = load_module(P.PolyAttention(dim=64, heads=4, dim_head=16), gd)
    b = lambda k: torch.as_tensor(gd[k]).cuda()  # noqa: E731
    with torch.no_grad():
        y = m(dev(gd["x"]), context=(dev(gd["c1"]), dev(gd["c2"])), mask=b("mx"), context_mask=(b("m1"), b("m2")))
    assert_close(y, gd["y"], torch.float32)


def test_order2_module_kv_cache_golden(golden):
    import poly_attention_b200 as P
    gd = golden("mod2_cache")
    m = load_module(P.PolyAttention(dim=64, heads=4, kv_heads=2, dim_head=16, causal=True), gd)
    x = dev(gd["x"])
    outs, cache = [], None
    with torch.no_grad():
        assert_close(m(x), gd["y"], torch.float32)
        for i in range(x.shape[1]):
            o, cache = m(x[:, i:i + 1], cache=cache, return_cache=True)
            outs.append(o)
    assert_close(torch.cat(outs, -2), gd["y_step"], torch.float32)
    for i, c in enumerate(cache):
        assert_close(c, gd[f"c{i}"], torch.float32, f"cache {i}")


@pytest.mark.parametrize("order", [3, 4])
@pytest.mark.parametrize("kvh", [4, 2])
def test_npoly_module_and_cache_golden(golden, order, kvh):
    import poly_attention_b200 as P
    gd = golden(f"modn_o{order}_g{kvh}")
    m = load_module(P.NPolyAttention(dim=64, order=order, heads=4, kv_heads=kvh, dim_head=16, causal=True,
                                     softclamp_value=20.0 if order == 3 else None), gd)
    x = dev(gd["x"])
    outs, cache = [], None
    with torch.no_grad():
        assert_close(m(x), gd["y"], torch.float32)
        for i in range(x.shape[1]):
            o, cache = m(x[:, i:i + 1], cache=cache, return_cache=True)
            outs.append(o)
    assert_close(torch.cat(outs, -2), gd["y_step"], torch.float32)
    c_qs, c_vs, c_lses, c_msgs = cache
    for i, t in enumerate(c_msgs):
        assert_close(t, gd[f"cmsg{i}"], torch.float32, f"msg cache {i}")


def test_lse_merge_equals_full_pass():
    import poly_attention_b200 as P
    b, h, n, d = 1, 2, 40, 64
    q, k, v = (dev(rnd((b, h, n, d), i)) for i in range(3))
    full, lse_full = P.pass_fwd(q, k, v)
    parts = [P.pass_fwd(q, k[:, :, s], v[:, :, s]) for s in (slice(0, 13), slice(13, 40))]
    out, lse = P.lse_merge(torch.stack([p[0] for p in parts]), torch.stack([p[1] for p in parts]))
    assert_close(out, host(full), torch.float32)
    assert_close(lse, host(lse_full), torch.float32)


@pytest.mark.parametrize("d", [64, 128])
@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("n", [300, 1024])
def test_tc_forward_selected_and_matches(d, causal, n):
    """bf16 / fp16 with d in {64, 128} must run the tcgen05 kernel."""
    import poly_attention_b200 as P
    for dtype in (torch.bfloat16, torch.float16):
        b, h, g = 1, 4, 2
        q = quant(rnd((b, h, n, d), 1), dtype)
        k, v = (quant(rnd((b, g, n, d), s), dtype) for s in (2, 3))
        bias = rnd((b, g, n), 4)
        qt, kt, vt = dev(q, dtype), dev(k, dtype), dev(v, dtype)
        assert P.kernel_names(qt, kt, vt, causal=causal)[0] == "tc100"
        out, lse = P.pass_fwd(qt, kt, vt, causal=causal, bias=dev(bias))
        eo, el = O.pass_fwd(q, np.repeat(k, 2, 1), np.repeat(v, 2, 1), causal=causal, bias=np.repeat(bias, 2, 1))
        assert_close(out, eo, dtype, f"out {dtype}")
        assert_close(lse, el, dtype, f"lse {dtype}")


@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("n,g", [(300, 2), (1024, 4)])
@pytest.mark.parametrize("softclamp", [None, 20.0])
@pytest.mark.parametrize("d", [64, 128])
def test_tc_backward_selected_and_matches(causal, n, g, softclamp, d):
    """bf16 / fp16 with d = 64 or 128 must run a tcgen05 backward; grads vs oracle."""
    import poly_attention_b200 as P
    b, h = 1, 4
    r = h // g
    for dtype in (torch.bfloat16, torch.float16):
        q = quant(rnd((b, h, n, d), 1), dtype)
        k, v = (quant(rnd((b, g, n, d), s), dtype) for s in (2, 3))
        do = quant(rnd((b, h, n, d), 4), dtype)
        bias = rnd((b, g, n), 5)
        dlse = rnd((b, h, n), 6)
        qt, kt, vt = dev(q, dtype), dev(k, dtype), dev(v, dtype)
        assert P.kernel_names(qt, kt, vt, causal=causal)[1] == "tc100"
        out, lse = P.pass_fwd(qt, kt, vt, causal=causal, softclamp=softclamp, bias=dev(bias))
        dq, dk, dv, db = P.pass_bwd(qt, kt, vt, out, lse, dev(do, dtype), causal=causal, softclamp=softclamp,
                                    bias=dev(bias), dlse=dev(dlse), want_dbias=True)
        edq, edk, edv, edb = O._pass_bwd(q, np.repeat(k, r, 1), np.repeat(v, r, 1), do, scale=d ** -0.5,
                                         causal=causal, softclamp_value=softclamp, key_mask=None, query_mask=None,
                                         bias=np.repeat(bias, r, 1), dlse=dlse)
        group = lambda t: t.reshape(b, g, r, *t.shape[2:]).sum(2)  # noqa: E731
        assert_close(dq, edq, dtype, f"dq {dtype}")
        assert_close(dk, group(edk), dtype, f"dk {dtype}")
        assert_close(dv, group(edv), dtype, f"dv {dtype}")
        # dbias_j = sum_i p_ij (dp_ij - delta_i): delta_i = dout_i . out_i uses the
        # 16-bit forward output (relative error ~2^-8), so the bound grows with the
        # column mass sum_i p_ij of key j.
        _, lse_ref = O.pass_fwd(q, np.repeat(k, r, 1), np.repeat(v, r, 1), causal=causal,
                                softclamp_value=softclamp, bias=np.repeat(bias, r, 1))
        s_ = np.einsum("bhid,bhjd->bhij", q, np.repeat(k, r, 1)) * d ** -0.5
        if softclamp:
            s_ = softclamp * np.tanh(s_ / softclamp)
        s_ = s_ + np.repeat(bias, r, 1)[..., None, :]
        if causal:
            s_ = np.where(np.triu(np.ones((n, n), bool), 1), -np.inf, s_)
        mass = group(np.exp(s_ - lse_ref[..., None]).sum(-2))
        err = np.abs(host(db) - group(edb))
        bound = BF16_ATOL + BF16_RTOL * np.abs(group(edb)) + 4e-3 * mass
        assert np.all(err <= bound), f"dbias {dtype}: worst excess {float((err - bound).max())}"


@pytest.mark.parametrize("nq,nk", [(384, 300), (128, 200), (300, 384), (257, 129)])
@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("d", [64, 128])
def test_tc_ragged_without_bias(nq, nk, causal, d):
    """Ragged key tails without a bias take the kernels' tail-masking path."""
    import poly_attention_b200 as P
    dtype = torch.bfloat16
    q = quant(rnd((1, 2, nq, d), 1), dtype)
    k, v = (quant(rnd((1, 2, nk, d), s), dtype) for s in (2, 3))
    do = quant(rnd((1, 2, nq, d), 4), dtype)
    qt, kt, vt = dev(q, dtype), dev(k, dtype), dev(v, dtype)
    assert P.kernel_names(qt, kt, vt, causal=causal) == ("tc100", "tc100")
    out, lse = P.pass_fwd(qt, kt, vt, causal=causal)
    eo, el = O.pass_fwd(q, k, v, causal=causal)
    assert_close(out, eo, dtype, "out")
    assert_close(lse, el, dtype, "lse")
    dq, dk, dv, _ = P.pass_bwd(qt, kt, vt, out, lse, dev(do, dtype), causal=causal)
    e = O._pass_bwd(q, k, v, do, scale=d ** -0.5, causal=causal, softclamp_value=None, key_mask=None,
                    query_mask=None, bias=None)
    assert_close(dq, e[0], dtype, "dq")
    assert_close(dk, e[1], dtype, "dk")
    assert_close(dv, e[2], dtype, "dv")


@pytest.mark.parametrize("order", [2, 3])
def test_polyvit_golden(golden, order):
    """PolyViT forward (poly_attention/poly_vit.py:65-101) vs the reference, fp32."""
    import poly_attention_b200 as P
    gd = golden(f"vit_o{order}")
    m = P.PolyViT(image_size=32, patch_size=8, num_classes=10, dim=64, depth=2, heads=4, mlp_dim=128, dim_head=16,
                  order=order)
    m = load_module(m, gd)
    with torch.no_grad():
        y = m(dev(gd["img"]))
    assert_close(y, gd["y"], torch.float32)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("d", [32, 128])
def test_pass_bwd_other_head_dims(dtype, d):
    """Backward at other head sizes: d = 32 (and fp32) on the CUDA cores, d = 128
    bf16 on the head_dim-128 tcgen05 kernel (70 rows: one partial tile)."""
    import poly_attention_b200 as P
    b, h, g, n = 1, 4, 2, 70
    q = quant(rnd((b, h, n, d), 1), dtype)
    k, v = (quant(rnd((b, g, n, d), s), dtype) for s in (2, 3))
    do = quant(rnd((b, h, n, d), 4), dtype)
    qt, kt, vt = dev(q, dtype), dev(k, dtype), dev(v, dtype)
    assert P.kernel_names(qt, kt, vt, causal=True)[1] == ("tc100" if d == 128 and dtype != torch.float32 else "simt")
    out, lse = P.pass_fwd(qt, kt, vt, causal=True)
    dq, dk, dv, _ = P.pass_bwd(qt, kt, vt, out, lse, dev(do, dtype), causal=True)
    r = h // g
    e = O._pass_bwd(q, np.repeat(k, r, 1), np.repeat(v, r, 1), do, scale=d ** -0.5, causal=True,
                    softclamp_value=None, key_mask=None, query_mask=None, bias=None)
    group = lambda t: t.reshape(b, g, r, *t.shape[2:]).sum(2)  # noqa: E731
    assert_close(dq, e[0], dtype, "dq")
    assert_close(dk, group(e[1]), dtype, "dk")
    assert_close(dv, group(e[2]), dtype, "dv")


@pytest.mark.parametrize("causal", [False, True])
def test_order2_pass1_mask_fully_masking_a_sequence(causal):
    """context_mask = (None, cm2) with one sequence fully masked in pass 1:
    its lse23 rows are -finfo.max, so pass 2 sees only dead keys there and must
    give the reference's uniform average (the routing sends pass 2 to the
    masked-pass kernels)."""
    import poly_attention_b200 as P
    dtype = torch.bfloat16
    b, h, n, d = 2, 2, 96, 64
    q1, q2, q3, v3 = (quant(rnd((b, h, n, d), s), dtype) for s in (31, 32, 33, 34))
    cm2 = np.ones((b, n), dtype=bool)
    cm2[1] = False
    cm2[0, 40:] = False
    out, _, _ = P.poly_attention_order2(dev(q1, dtype), dev(q2, dtype), dev(q3, dtype), dev(v3, dtype),
                                        context_mask=(None, torch.as_tensor(cm2).cuda()), causal=causal)
    eo, _, _ = O.order2_fwd(q1, q2, q2, q3, v3, context_mask=(None, cm2), causal=causal)
    assert_close(out, eo, dtype, "out")


@pytest.mark.parametrize("d", [64, 128])
@pytest.mark.parametrize("off,nq,nk", [(128, 256, 384), (256, 300, 556), (512, 128, 600)])
def test_pass_fwd_causal_offset(d, off, nq, nk):
    """causal_offset: the queries are rows [off, off + nq) of the key sequence
    (key j visible iff j <= i + off); equals the oracle's top-left causal pass
    over the whole sequence, restricted to those rows."""
    import poly_attention_b200 as P
    b, h = 2, 4
    dt = torch.bfloat16
    qf = quant(rnd((b, h, off + nq, d), 1), dt)
    k, v = (quant(rnd((b, h, nk, d), i + 2), dt) for i in range(2))
    bias = rnd((b, h, nk), 9)
    out, lse = P.pass_fwd(dev(qf[:, :, off:], dt), dev(k, dt), dev(v, dt), causal=True, bias=dev(bias),
                          causal_offset=off)
    assert P.kernel_names(dev(qf[:, :, off:], dt), dev(k, dt), dev(v, dt), causal=True)[0] == "tc100"
    eo, el = O.pass_fwd(qf, k, v, causal=True, bias=bias)
    assert_close(out, eo[:, :, off:], dt, "out")
    assert_close(lse, el[:, :, off:], dt, "lse")


def test_pass_fwd_causal_offset_rejected_where_unsupported():
    import poly_attention_b200 as P
    q = torch.randn(1, 2, 256, 64, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(Exception):
        P.pass_fwd(q, q, q, causal=True, causal_offset=100)        # not a multiple of 128
    with pytest.raises(Exception):
        P.pass_fwd(q.float(), q.float(), q.float(), causal=True, causal_offset=128)   # fp32 kernel
