"""The order-2 core as torch.library custom ops: opcheck (schema, fake
shapes, autograd registration) and the module under torch.compile inside an
autocast region, as the reference's test_compile_poly_attention
(tests/test_poly_attention.py:275-289) runs it (without rotary: its package
is not installed here), against the same module run eagerly."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_order2_ops_opcheck():
    import poly_attention_b200  # noqa: F401  (registers the ops)
    g = torch.Generator(device="cuda").manual_seed(0)
    mk = lambda h: torch.randn(2, h, 48, 32, device="cuda", generator=g).requires_grad_(True)  # noqa: E731
    args = (mk(4), mk(2), mk(2), mk(2), None, None, None, None, 0.0, True)
    torch.library.opcheck(torch.ops.poly_b200.order2_fwd, args)
    args_sc = (mk(2), mk(2), mk(2), mk(2), mk(2), None, None, None, 20.0, False)
    torch.library.opcheck(torch.ops.poly_b200.order2_fwd, args_sc)


@pytest.mark.parametrize("causal", [False, True])
def test_compiled_module_under_autocast_matches_eager(causal):
    from poly_attention_b200 import PolyAttention
    torch.manual_seed(0)
    attn = PolyAttention(dim=128, heads=4, dim_head=64, causal=causal).cuda()
    x = torch.randn(2, 64, 128, device="cuda")
    xe, xc = x.clone().requires_grad_(True), x.clone().requires_grad_(True)
    with torch.autocast("cuda", dtype=torch.bfloat16):
        oe = attn(xe)
        oe.float().sum().backward()
    torch._dynamo.reset()
    model = torch.compile(attn, fullgraph=True)
    with torch.autocast("cuda", dtype=torch.bfloat16):
        oc = model(xc)
        oc.float().sum().backward()
    assert oc.shape == (2, 64, 128)
    assert not torch.isnan(oc).any()
    torch.testing.assert_close(oc.float(), oe.float(), atol=2e-2, rtol=1e-2)
    torch.testing.assert_close(xc.grad, xe.grad, atol=2e-2, rtol=1e-2)


def test_compiled_npoly_under_autocast_matches_eager():
    """The order-n module compiles (the chain core is an autograd Function:
    dynamo treats its library calls as graph breaks) and matches eager."""
    from poly_attention_b200 import NPolyAttention
    torch.manual_seed(1)
    attn = NPolyAttention(dim=128, order=3, heads=4, kv_heads=2, dim_head=64, causal=True).cuda()
    x = torch.randn(2, 96, 128, device="cuda")
    xe, xc = x.clone().requires_grad_(True), x.clone().requires_grad_(True)
    with torch.autocast("cuda", dtype=torch.bfloat16):
        oe = attn(xe)
        oe.float().sum().backward()
    torch._dynamo.reset()
    model = torch.compile(attn)
    with torch.autocast("cuda", dtype=torch.bfloat16):
        oc = model(xc)
        oc.float().sum().backward()
    torch.testing.assert_close(oc.float(), oe.float(), atol=2e-2, rtol=1e-2)
    torch.testing.assert_close(xc.grad, xe.grad, atol=2e-2, rtol=1e-2)
