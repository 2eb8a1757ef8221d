"""Pin the numpy oracle against golden vectors produced by the reference.

The vectors come from ``tests/golden/make_golden.py``, which runs the
reference PyTorch path (poly_attention/poly_attention.py:48-116,120-365 and
n_poly_attention.py:122-340) on CPU. CPU only.
"""
import numpy as np
import pytest

from oracle import poly_oracle as O

ATOL = 2e-5


def close(a, b, atol=ATOL, rtol=1e-4):
    np.testing.assert_allclose(a, b, atol=atol, rtol=rtol)


@pytest.mark.parametrize("n", (17, 64))
@pytest.mark.parametrize("causal", (0, 1))
@pytest.mark.parametrize("sc", (0, 20))
def test_reference_fn_fwd_bwd(golden, n, causal, sc):
    g = golden(f"ref_fn_n{n}_c{causal}_s{sc}")
    scv = None if sc == 0 else float(sc)
    out, lse, msg = O.order2_fwd(g["q1"], g["q2a"], g["q2b"], g["q3"], g["v3"], softclamp_value=scv, causal=bool(causal))
    close(out, g["out"]); close(lse, g["lse23"]); close(msg, g["msg"])
    grads = O.order2_bwd(g["q1"], g["q2a"], g["q2b"], g["q3"], g["v3"], g["dout"], softclamp_value=scv, causal=bool(causal))
    for name, gr in zip(("dq1", "dq2a", "dq2b", "dq3", "dv3"), grads):
        close(gr, g[name], atol=1e-4)


@pytest.mark.parametrize("causal", (0, 1))
def test_reference_fn_masked(golden, causal):
    g = golden(f"ref_fn_masked_c{causal}")
    cm = (g["cm1"], g["cm2"])
    out, lse, msg = O.order2_fwd(g["q1"], g["q2a"], g["q2b"], g["q3"], g["v3"], mask=g["mask"], context_mask=cm,
                                 causal=bool(causal))
    close(out, g["out"]); close(lse, g["lse23"]); close(msg, g["msg"])
    grads = O.order2_bwd(g["q1"], g["q2a"], g["q2b"], g["q3"], g["v3"], g["dout"], mask=g["mask"], context_mask=cm,
                         causal=bool(causal))
    for name, gr in zip(("dq1", "dq2a", "dq2b", "dq3", "dv3"), grads):
        close(gr, g[name], atol=1e-4)


def test_reference_fn_cache(golden):
    g = golden("ref_fn_cache")
    q2f = np.concatenate([g["cq2"], g["q2"]], -2)
    q3f = np.concatenate([g["cq3"], g["q3"]], -2)
    v3f = np.concatenate([g["cv3"], g["v3"]], -2)
    out, lse, msg = O.order2_fwd(g["q1"], g["q2"], q2f, q3f, v3f, causal=True,
                                 cache=(g["cq2"], g["cq3"], g["cv3"], g["clse"], g["cmsg"]))
    close(out, g["out"]); close(lse, g["lse23"]); close(msg, g["msg"])


MOD2 = {
    "base": dict(heads=4),
    "causal_gqa": dict(heads=4, kv_heads=2, causal=True, softclamp_value=20.0),
    "root_gate": dict(heads=4, causal=True, multiply_root_value=True, use_root_value_as_attn_gate=True, attn_gate=True),
    "shared_prenorm": dict(heads=4, kv_heads=1, shared_kv=True, prenorm=True, multiply_root_value=True),
}


def params(g):
    return {k[2:]: v for k, v in g.items() if k.startswith("p:")}


@pytest.mark.parametrize("name", sorted(MOD2))
def test_order2_module(golden, name):
    g = golden(f"mod2_{name}")
    y = O.order2_module_fwd(params(g), g["x"], **MOD2[name])
    close(y, g["y"])


def test_order2_module_context_masks(golden):
    g = golden("mod2_context_masks")
    y = O.order2_module_fwd(params(g), g["x"], heads=4, context=(g["c1"], g["c2"]), mask=g["mx"],
                            context_mask=(g["m1"], g["m2"]))
    close(y, g["y"])


def test_order2_module_cache(golden):
    g = golden("mod2_cache")
    p = params(g)
    kw = dict(heads=4, kv_heads=2, causal=True)
    close(O.order2_module_fwd(p, g["x"], **kw), g["y"])
    cache, outs = None, []
    for i in range(g["x"].shape[1]):
        o, cache = O.order2_module_fwd(p, g["x"][:, i:i + 1], cache=cache, return_cache=True, **kw)
        outs.append(o)
    close(np.concatenate(outs, -2), g["y_step"])
    for i, c in enumerate(cache):
        if c.shape == g[f"c{i}"].shape:
            close(c, g[f"c{i}"])
        else:  # lse / msg caches: the reference keeps them at query-head width
            r = g[f"c{i}"].shape[1] // c.shape[1]
            close(np.repeat(c, r, axis=1), g[f"c{i}"])


@pytest.mark.parametrize("order", (3, 4))
@pytest.mark.parametrize("kvh", (4, 2))
def test_npoly_module_and_cache(golden, order, kvh):
    g = golden(f"modn_o{order}_g{kvh}")
    p = params(g)
    kw = dict(order=order, heads=4, kv_heads=kvh, causal=True, softclamp_value=20.0 if order == 3 else None)
    close(O.npoly_module_fwd(p, g["x"], **kw), g["y"])
    cache, outs = None, []
    for i in range(g["x"].shape[1]):
        o, cache = O.npoly_module_fwd(p, g["x"][:, i:i + 1], cache=cache, return_cache=True, **kw)
        outs.append(o)
    close(np.concatenate(outs, -2), g["y_step"])
    c_qs, c_vs, c_lses, c_msgs = cache
    for i, t in enumerate(c_qs):
        close(t, g[f"cq{i}"])
    for i, t in enumerate(c_lses):
        close(t, g[f"clse{i}"], atol=1e-4)
    for i, t in enumerate(c_msgs):
        close(t, g[f"cmsg{i}"])


@pytest.mark.parametrize("order", (2, 3, 4))
def test_chain_gradients(golden, order):
    g = golden(f"chain_grad_o{order}")
    qs = [g[f"q{i}"] for i in range(order + 1)]
    vs = [g[f"v{i}"] for i in range(2, order + 1)]   # v3..v_{order+1}
    sc = 20.0 if order == 3 else None
    out, _, _ = O.npoly_chain_fwd(qs[:-1], qs[1:], vs, causal=True, softclamp_value=sc)
    close(out, g["chain_out"])
    dql, dqr, dvs = O.npoly_chain_bwd(qs[:-1], qs[1:], vs, g["dchain"], causal=True, softclamp_value=sc)
    # q_t (t >= 1) is the key of score t-1 and the query of score t
    dq = [dql[0]] + [dqr[t - 1] + (dql[t] if t < order else 0) for t in range(1, order + 1)]
    for i in range(order + 1):
        close(dq[i], g[f"dq{i}"], atol=1e-4)
    for i, dv in enumerate(dvs):
        close(dv, g[f"dv{i + 2}"], atol=1e-4)
