"""GPU parity of the fp32 pass on the tensor cores (3xTF32, mma.sync) against
the numpy oracle at the fp32 bar (1e-4): config 1's shape, ragged sizes,
causal, per-key bias with dead keys, fully dead rows (the reference's
uniform-average result), softclamp, GQA."""
import numpy as np
import pytest
import torch

from oracle import poly_oracle as O

pytestmark = pytest.mark.gpu
TOL = 1e-4


def rnd(shape, seed):
    return np.random.default_rng(seed).standard_normal(shape).astype(np.float32)


def dev(a):
    return torch.as_tensor(np.ascontiguousarray(a)).cuda()


@pytest.mark.parametrize("b,h,g,nq,nk", [(1, 8, 8, 1024, 1024), (2, 4, 2, 100, 77), (1, 2, 1, 300, 513)])
@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("extras", ["none", "bias", "bias+softclamp"])
def test_f32_pass(b, h, g, nq, nk, causal, extras):
    import poly_attention_b200 as P
    d = 64
    q = rnd((b, h, nq, d), 1)
    k, v = rnd((b, g, nk, d), 2), rnd((b, g, nk, d), 3)
    kw, okw = {}, {}
    if "bias" in extras:
        bias = rnd((b, g, nk), 4)
        bias[:, :, 3::11] = -np.finfo(np.float32).max
        kw["bias"], okw["bias"] = dev(bias), np.repeat(bias, h // g, 1)
    if "softclamp" in extras:
        kw["softclamp"], okw["softclamp_value"] = 20.0, 20.0
    qt, kt, vt = dev(q), dev(k), dev(v)
    assert P.kernel_names(qt, kt, vt, causal=causal)[0] == "tf32x3"
    out, lse = P.pass_fwd(qt, kt, vt, causal=causal, **kw)
    eo, el = O.pass_fwd(q, np.repeat(k, h // g, 1), np.repeat(v, h // g, 1), causal=causal, **okw)
    np.testing.assert_allclose(out.cpu().numpy(), eo, atol=TOL, rtol=TOL)
    np.testing.assert_allclose(lse.cpu().numpy(), el, atol=TOL, rtol=TOL)


@pytest.mark.parametrize("causal", [False, True])
def test_f32_pass_fully_dead_rows(causal):
    """Every key dead for one sequence: the reference's -finfo.max arithmetic
    gives a uniform average over the keys not both masked and dead."""
    import poly_attention_b200 as P
    b, h, n, d = 2, 2, 70, 64
    q, k, v = rnd((b, h, n, d), 5), rnd((b, h, n, d), 6), rnd((b, h, n, d), 7)
    bias = rnd((b, h, n), 8)
    bias[1] = -np.finfo(np.float32).max
    out, lse = P.pass_fwd(dev(q), dev(k), dev(v), causal=causal, bias=dev(bias))
    eo, el = O.pass_fwd(q, k, v, causal=causal, bias=bias)
    np.testing.assert_allclose(out.cpu().numpy(), eo, atol=TOL, rtol=TOL)
    np.testing.assert_allclose(lse.cpu().numpy(), el, atol=TOL, rtol=TOL)
