"""GPU parity of the short-sequence pass kernel (seq_q, seq_k <= 128: one CTA
per (batch, head), mma.sync tiles, exact row softmax) against the numpy
oracle: causal and not, per-key bias with dead keys, softclamp, GQA, ragged
sizes, bf16 and fp16, head sizes 64 and 128."""
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


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("d", [64, 128])
@pytest.mark.parametrize("nq,nk", [(64, 64), (37, 100), (128, 128), (100, 7), (2, 128), (17, 17)])
@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("extras", ["none", "bias", "bias+softclamp"])
def test_small_pass(dt, d, nq, nk, causal, extras):
    import poly_attention_b200 as P
    b, h, g = 3, 4, 2
    q = host(dev(rnd((b, h, nq, d), 1), dt))
    k, v = (host(dev(rnd((b, g, nk, d), s), dt)) for s in (2, 3))
    bias = rnd((b, g, nk), 4)
    bias[:, :, 5::9] = -np.finfo(np.float32).max            # dead keys (a fully masked previous row)
    kw, okw = {}, {}
    if "bias" in extras:
        kw["bias"] = dev(bias, torch.float32)
        okw["bias"] = np.repeat(bias, h // g, 1)
    if "softclamp" in extras:
        kw["softclamp"] = 20.0
        okw["softclamp_value"] = 20.0
    qt, kt, vt = dev(q, dt), dev(k, dt), dev(v, dt)
    assert P.kernel_names(qt, kt, vt, causal=causal)[0] == "small"
    out, lse = P.pass_fwd(qt, kt, vt, causal=causal, **kw)
    eo, el = O.pass_fwd(q, np.repeat(k, h // g, 1), np.repeat(v, h // g, 1), causal=causal, **okw)
    np.testing.assert_allclose(host(out), eo, atol=ATOL, rtol=RTOL)
    np.testing.assert_allclose(host(lse), el, atol=ATOL, rtol=RTOL)


def test_small_pass_strided_inputs():
    """Head-split views of projection outputs (the module path) without copies."""
    import poly_attention_b200 as P
    b, h, n, d, dt = 2, 4, 64, 64, torch.bfloat16
    qkv = torch.randn(b, n, 3, h, d, device="cuda", dtype=dt)
    q, k, v = qkv.permute(2, 0, 3, 1, 4)
    assert P.kernel_names(q, k, v)[0] == "small"
    out, lse = P.pass_fwd(q, k, v)
    qf, kf, vf = (host(t.contiguous()) for t in (q, k, v))
    eo, el = O.pass_fwd(qf, kf, vf)
    np.testing.assert_allclose(host(out), eo, atol=ATOL, rtol=RTOL)
    np.testing.assert_allclose(host(lse), el, atol=ATOL, rtol=RTOL)


@pytest.mark.parametrize("causal", [False, True])
def test_small_pass_fully_dead_rows(causal):
    """Every key dead for one sequence: the reference's uniform-average result
    (keys both causally masked and dead drop out), lse = -FLT_MAX."""
    import poly_attention_b200 as P
    dt = torch.bfloat16
    b, h, n, d = 2, 2, 50, 64
    q, k, v = (host(dev(rnd((b, h, n, d), s), dt)) for s in (5, 6, 7))
    bias = rnd((b, h, n), 8)
    bias[1] = -np.finfo(np.float32).max
    out, lse = P.pass_fwd(dev(q, dt), dev(k, dt), dev(v, dt), causal=causal, bias=dev(bias, torch.float32))
    eo, el = O.pass_fwd(q, k, v, causal=causal, bias=bias)
    np.testing.assert_allclose(host(out), eo, atol=ATOL, rtol=RTOL)
    np.testing.assert_allclose(host(lse), el, atol=ATOL, rtol=RTOL)
