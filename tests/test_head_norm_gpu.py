"""poly_head_rmsnorm (the modules' q_norms, read from strided head-split
views, one launch per layer) against nn.RMSNorm applied tensor by tensor:
values, output dtype and eps rule (module eps, or finfo eps), inside and
outside autocast, and gradients through the registered autograd."""
import pytest
import torch
from torch import nn

pytestmark = pytest.mark.gpu


def _views(dt, d, heads=(4, 2, 2)):
    # projection outputs [b, n, (h d)] split into [b, h, n, d] strided views, as split_heads makes them
    b, n = 3, 37
    xs = []
    for h in heads:
        t = torch.randn(b, n, 2 * h * d, device="cuda", dtype=dt)
        xs.append(t.view(b, n, 2, h, d).permute(2, 0, 3, 1, 4)[1])
    return xs


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("d", [64, 128, 32])
@pytest.mark.parametrize("eps", [None, 1e-6])
def test_head_rmsnorm_matches_rmsnorm(dt, d, eps):
    from poly_attention_b200.head_norm import head_rmsnorm
    norms = [nn.RMSNorm(d, eps=eps).cuda().to(dt) for _ in range(3)]
    for nm in norms:
        nn.init.normal_(nm.weight, 1.0, 0.2)
    xs = _views(dt, d)
    got = head_rmsnorm(norms, xs)
    for g, nm, x in zip(got, norms, xs):
        ref = nm(x)
        assert g.dtype == ref.dtype and g.shape == ref.shape and g.is_contiguous()
        atol, rtol = (1e-5, 1e-5) if dt == torch.float32 else (2e-2, 1e-2)   # 16-bit: rounding order
        torch.testing.assert_close(g.float(), ref.float(), atol=atol, rtol=rtol)


def test_head_rmsnorm_autocast_and_fp32_weights():
    from poly_attention_b200.head_norm import head_rmsnorm
    d = 64
    norms = [nn.RMSNorm(d).cuda() for _ in range(5)]     # fp32 weights, eps None, five tensors (two launches)
    for nm in norms:
        nn.init.normal_(nm.weight, 1.0, 0.2)
    xs = _views(torch.bfloat16, d, heads=(4, 2, 2, 2, 2))
    with torch.autocast("cuda", dtype=torch.bfloat16):
        got = head_rmsnorm(norms, xs)
        refs = [nm(x) for nm, x in zip(norms, xs)]
    for g, r in zip(got, refs):
        assert g.dtype == r.dtype
        torch.testing.assert_close(g.float(), r.float(), atol=2e-2, rtol=1e-2)
    got = head_rmsnorm(norms, xs)                         # outside autocast: bf16 x, fp32 weight
    for g, nm, x in zip(got, norms, xs):
        r = nm(x)
        assert g.dtype == r.dtype
        torch.testing.assert_close(g.float(), r.float(), atol=2e-2, rtol=1e-2)


def test_head_rmsnorm_gradients():
    from poly_attention_b200.head_norm import head_rmsnorm
    d = 64
    norms = [nn.RMSNorm(d).cuda() for _ in range(3)]
    for nm in norms:
        nn.init.normal_(nm.weight, 1.0, 0.2)
    xs = [x.float().detach().requires_grad_(True) for x in _views(torch.float32, d)]
    xr = [x.detach().clone().requires_grad_(True) for x in xs]
    gs = [torch.randn(x.shape, device="cuda") for x in xs]
    got = head_rmsnorm(norms, xs)
    torch.autograd.backward(got, gs)
    gw = [nm.weight.grad.clone() for nm in norms]
    for nm in norms:
        nm.weight.grad = None
    torch.autograd.backward([nm(x) for nm, x in zip(norms, xr)], gs)
    for a, b in zip(xs, xr):
        torch.testing.assert_close(a.grad, b.grad, atol=1e-4, rtol=1e-4)
    for a, nm in zip(gw, norms):
        torch.testing.assert_close(a, nm.weight.grad, atol=1e-3, rtol=1e-4)
