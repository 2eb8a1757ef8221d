"""GPU test of HostStreamedOrder2 (host tensors in, gradients out, batch
chunks streamed over three CUDA streams) against the device-resident autograd
path of flash_poly_attention on the same inputs: same kernels, so the only
difference allowed is fp32 summation order in the dQ reduction."""
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("b,h,g,n,chunk,slots", [(4, 4, 2, 384, 1, 3), (6, 2, 2, 256, 2, 2), (3, 4, 4, 200, 1, 1)])
def test_host_streamed_step_matches_device_autograd(b, h, g, n, chunk, slots):
    import poly_attention_b200 as P
    d, dt = 64, torch.bfloat16
    gen = torch.Generator().manual_seed(5)
    hq = [torch.randn(b, h, n, d, generator=gen).to(dt).pin_memory()]
    hk = [torch.randn(b, g, n, d, generator=gen).to(dt).pin_memory() for _ in range(3)]
    hdo = torch.randn(b, h, n, d, generator=gen).to(dt).pin_memory()
    hosts = hq + hk + [hdo]
    st = P.HostStreamedOrder2(batch=b, heads=h, kv_heads=g, seq_len=n, dim_head=d, chunk=chunk, slots=slots)
    out_h = torch.empty(b, h, n, d, dtype=dt).pin_memory()
    for _ in range(2):                      # twice: slot reuse across steps
        grads = st.step(*hosts, out=out_h)
        torch.cuda.synchronize()
    ts = [x.cuda().requires_grad_(True) for x in hosts[:4]]
    out = P.flash_poly_attention(*ts, is_causal=True)
    out.backward(hdo.cuda())
    torch.testing.assert_close(out_h, out.detach().cpu(), atol=0, rtol=0)
    for gh, tt in zip(grads, ts):
        torch.testing.assert_close(gh.float(), tt.grad.float().cpu(), atol=2e-2, rtol=1e-2)


def test_host_streamed_refuses_device_tensors():
    import poly_attention_b200 as P
    st = P.HostStreamedOrder2(batch=1, heads=1, kv_heads=1, seq_len=64, dim_head=64)
    x = torch.zeros(1, 1, 64, 64, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(ValueError):
        st.step(x, x, x, x, x)


def test_host_streamed_overlapping_steps():
    """sync=False steps overlap across step boundaries (slots are reused only
    after their previous chunk computed); after join() every step's gradients
    equal those of synchronous steps."""
    import poly_attention_b200 as P
    b, h, n, d, dt = 4, 2, 256, 64, torch.bfloat16
    gen = torch.Generator().manual_seed(6)
    batches = [[torch.randn(b, h, n, d, generator=gen).to(dt).pin_memory() for _ in range(5)] for _ in range(3)]
    st = P.HostStreamedOrder2(batch=b, heads=h, kv_heads=h, seq_len=n, dim_head=d, chunk=1, slots=2)
    outs = [[torch.empty(b, h, n, d, dtype=dt).pin_memory() for _ in range(4)] for _ in batches]
    for x, g in zip(batches, outs):
        st.step(*x, grads=g, sync=False)
    st.join()
    torch.cuda.synchronize()
    for x, g in zip(batches, outs):
        ref = st.step(*x)
        torch.cuda.synchronize()
        for a, r in zip(g, ref):
            torch.testing.assert_close(a.float(), r.float(), atol=2e-2, rtol=1e-2)
