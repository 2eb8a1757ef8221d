"""Generate golden vectors by running the reference implementation itself.

Run where a checkout of lucidrains/poly-attention (read-only) is available,
with ``POLY_REFERENCE`` naming its directory:

    POLY_REFERENCE=<checkout> python tests/golden/make_golden.py

The three dependencies the reference imports but this image lacks (einx,
torch-einops-utils, rotary-embedding-torch) are replaced by the test-only
shims in ``tests/golden/shims`` (each implements only the call-site patterns,
rotary is a non-functional stub). Everything else is the reference's own code
and torch. Outputs are small float32 ``.npz`` files in this folder; they are
committed, and nothing on a GPU box needs the reference.

Cases (all fp32, CPU, seeded):

* ``ref_fn_*``   ``reference_poly_attention`` forward + autograd backward
  (poly_attention/poly_attention.py:48-116), causal x softclamp, two lengths,
  plus masked and cached variants.
* ``mod2_*``     ``Order2PolyAttention`` module forward with its state_dict
  (poly_attention/poly_attention.py:120-365), GQA / root value / gates /
  shared kv variants, and a stepwise-cache run.
* ``modn_*``     ``NPolyAttention`` order 3 and 4 forward (n_poly_attention.py),
  with a stepwise-cache run, plus chain-level gradients captured with hooks
  on the q-norm outputs, the kv projections and the output projection input.
* ``vit_*``      ``PolyViT`` forward, small; ``vit_full``: the full config-3
  model (dim 1024, depth 6) on 2 images, outputs only (weights and images
  come from seeds, tests/golden/seeded.py).

``python tests/golden/make_golden.py [case ...]`` regenerates only the named
case groups (ref_fn, mod2, modn, vit, vit_full).
"""
from __future__ import annotations

import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REF = os.environ.get("POLY_REFERENCE")
if not REF or not os.path.isdir(os.path.join(REF, "poly_attention")):
    sys.exit("set POLY_REFERENCE to a checkout of lucidrains/poly-attention (the directory holding poly_attention/)")
sys.path.insert(0, os.path.join(HERE, "shims"))
sys.path.insert(0, HERE)
sys.path.insert(0, REF)

from poly_attention.poly_attention import reference_poly_attention, Order2PolyAttention  # noqa: E402
from poly_attention.n_poly_attention import NPolyAttention  # noqa: E402
from poly_attention.poly_vit import PolyViT  # noqa: E402


def np32(t):
    return t.detach().cpu().numpy().astype(np.float32)


def save(name, **arrays):
    path = os.path.join(HERE, f"{name}.npz")
    np.savez_compressed(path, **arrays)
    print("wrote", path, sum(a.nbytes for a in arrays.values()), "bytes")


def ref_fn_cases():
    out = {}
    for n in (17, 64):
        for causal in (False, True):
            for sc in (None, 20.0):
                torch.manual_seed(1000 + n + 2 * causal + (sc is not None))
                shape = (2, 2, n, 32)
                ts = [torch.randn(shape, requires_grad=True) for _ in range(5)]
                q1, q2a, q2b, q3, v3 = ts
                o, lse, msg = reference_poly_attention(q1, q2a, q2b, q3, v3, softclamp_value=sc, causal=causal)
                do = torch.randn_like(o)
                o.backward(do)
                key = f"n{n}_c{int(causal)}_s{0 if sc is None else int(sc)}"
                out[key] = dict(q1=q1, q2a=q2a, q2b=q2b, q3=q3, v3=v3, out=o, lse23=lse, msg=msg, dout=do,
                                dq1=q1.grad, dq2a=q2a.grad, dq2b=q2b.grad, dq3=q3.grad, dv3=v3.grad)
    for key, d in out.items():
        save(f"ref_fn_{key}", **{k: np32(v) for k, v in d.items()})

    # masks: query mask + context masks, non-causal and causal
    for causal in (False, True):
        torch.manual_seed(77 + causal)
        n = 24
        shape = (2, 2, n, 32)
        ts = [torch.randn(shape, requires_grad=True) for _ in range(5)]
        q1, q2a, q2b, q3, v3 = ts
        mask = torch.ones(2, n, dtype=torch.bool)
        mask[0, 18:] = False
        mask[1, 5] = False
        cm1 = torch.ones(2, n, dtype=torch.bool)
        cm1[:, 20:] = False
        cm2 = torch.ones(2, n, dtype=torch.bool)
        cm2[0, 10:14] = False
        cm2[1, 0] = False          # row 0 fully masked in causal pass 1
        o, lse, msg = reference_poly_attention(q1, q2a, q2b, q3, v3, mask=mask, context_mask=(cm1, cm2),
                                               softclamp_value=None, causal=causal)
        do = torch.randn_like(o)
        o.backward(do)
        save(f"ref_fn_masked_c{int(causal)}", q1=np32(q1), q2a=np32(q2a), q2b=np32(q2b), q3=np32(q3), v3=np32(v3),
             mask=mask.numpy(), cm1=cm1.numpy(), cm2=cm2.numpy(), out=np32(o), lse23=np32(lse), msg=np32(msg),
             dout=np32(do), dq1=np32(q1.grad), dq2a=np32(q2a.grad), dq2b=np32(q2b.grad), dq3=np32(q3.grad),
             dv3=np32(v3.grad))

    # cache: one new position attending a cache of length L
    torch.manual_seed(5)
    L = 20
    b, h, d = 2, 2, 32
    cq2, cq3, cv3 = (torch.randn(b, h, L, d) for _ in range(3))
    clse = torch.randn(b, h, L)
    cmsg = torch.randn(b, h, L, d)
    q1, q2, q3, v3 = (torch.randn(b, h, 1, d) for _ in range(4))
    q2f, q3f, v3f = (torch.cat(p, -2) for p in ((cq2, q2), (cq3, q3), (cv3, v3)))
    o, lse, msg = reference_poly_attention(q1, q2, q2f, q3f, v3f, causal=True, cache=(cq2, cq3, cv3, clse, cmsg))
    save("ref_fn_cache", cq2=np32(cq2), cq3=np32(cq3), cv3=np32(cv3), clse=np32(clse), cmsg=np32(cmsg),
         q1=np32(q1), q2=np32(q2), q3=np32(q3), v3=np32(v3), out=np32(o), lse23=np32(lse), msg=np32(msg))


MOD2_VARIANTS = {
    "base": dict(heads=4),
    "causal_gqa": dict(heads=4, kv_heads=2, causal=True, softclamp_value=20.0),
    "root_gate": dict(heads=4, causal=True, multiply_root_value=True, use_root_value_as_attn_gate=True, attn_gate=True),
    "shared_prenorm": dict(heads=4, kv_heads=1, shared_kv=True, prenorm=True, multiply_root_value=True),
}


def state_np(mod):
    return {k: np32(v) for k, v in mod.state_dict().items()}


def mod2_cases():
    for name, cfg in MOD2_VARIANTS.items():
        torch.manual_seed(11)
        m = Order2PolyAttention(dim=64, dim_head=16, use_flash_kernel=False, **cfg)
        x = torch.randn(2, 12, 64)
        with torch.no_grad():
            y = m(x)
        arrays = {f"p:{k}": v for k, v in state_np(m).items()}
        save(f"mod2_{name}", x=np32(x), y=np32(y), **arrays)

    # masked + contexts of different lengths
    torch.manual_seed(12)
    m = Order2PolyAttention(dim=64, heads=4, dim_head=16, use_flash_kernel=False)
    x = torch.randn(2, 10, 64)
    c1, c2 = torch.randn(2, 13, 64), torch.randn(2, 15, 64)
    mx = torch.ones(2, 10, dtype=torch.bool); mx[:, 8:] = False
    m1 = torch.ones(2, 13, dtype=torch.bool); m1[:, 11:] = False
    m2 = torch.ones(2, 15, dtype=torch.bool); m2[:, 9:] = False
    with torch.no_grad():
        y = m(x, context=(c1, c2), mask=mx, context_mask=(m1, m2))
    save("mod2_context_masks", x=np32(x), c1=np32(c1), c2=np32(c2), mx=mx.numpy(), m1=m1.numpy(), m2=m2.numpy(),
         y=np32(y), **{f"p:{k}": v for k, v in state_np(m).items()})

    # stepwise cache (kv cache decode)
    torch.manual_seed(13)
    m = Order2PolyAttention(dim=64, heads=4, kv_heads=2, dim_head=16, causal=True, use_flash_kernel=False)
    x = torch.randn(2, 6, 64)
    outs = []
    cache = None
    with torch.no_grad():
        y_par = m(x)
        for i in range(6):
            o, cache = m(x[:, i:i + 1], cache=cache, return_cache=True)
            outs.append(o)
    save("mod2_cache", x=np32(x), y=np32(y_par), y_step=np32(torch.cat(outs, -2)),
         **{f"c{i}": np32(c) for i, c in enumerate(cache)}, **{f"p:{k}": v for k, v in state_np(m).items()})


def modn_cases():
    for order in (3, 4):
        for kvh in (4, 2):
            torch.manual_seed(20 + order + kvh)
            m = NPolyAttention(dim=64, order=order, heads=4, kv_heads=kvh, dim_head=16, causal=True,
                               softclamp_value=20.0 if order == 3 else None)
            x = torch.randn(2, 9, 64)
            outs = []
            cache = None
            with torch.no_grad():
                y = m(x)
                for i in range(9):
                    o, cache = m(x[:, i:i + 1], cache=cache, return_cache=True)
                    outs.append(o)
            c_qs, c_vs, c_lses, c_msgs = cache
            arrays = {f"p:{k}": v for k, v in state_np(m).items()}
            arrays.update({f"cq{i}": np32(t) for i, t in enumerate(c_qs)})
            arrays.update({f"cv{i}": np32(t) for i, t in enumerate(c_vs)})
            arrays.update({f"clse{i}": np32(t) for i, t in enumerate(c_lses)})
            arrays.update({f"cmsg{i}": np32(t) for i, t in enumerate(c_msgs)})
            save(f"modn_o{order}_g{kvh}", x=np32(x), y=np32(y), y_step=np32(torch.cat(outs, -2)), **arrays)

    # chain-level gradients (no GQA so q-norm outputs are exactly the chain inputs)
    for order in (2, 3, 4):
        torch.manual_seed(40 + order)
        m = NPolyAttention(dim=64, order=order, heads=4, dim_head=16, causal=True,
                           softclamp_value=20.0 if order == 3 else None)
        caps = {}

        def keep(name):
            def hook(mod, inp, out):
                out.retain_grad()
                caps[name] = out
            return hook

        for i, nm in enumerate(m.q_norms):
            nm.register_forward_hook(keep(f"qn{i}"))
        for i, lin in enumerate(m.to_kvs):
            lin.register_forward_hook(keep(f"kv{i}"))

        def pre(mod, args):
            args[0].retain_grad()
            caps["merged"] = args[0]
        m.to_out.register_forward_pre_hook(pre)

        x = torch.randn(2, 11, 64)
        y = m(x)
        dy = torch.randn_like(y)
        y.backward(dy)
        b, n = 2, 11
        arrays = {"dchain": np32(caps["merged"].grad.reshape(b, n, 4, 16).transpose(1, 2)),
                  "chain_out": np32(caps["merged"].reshape(b, n, 4, 16).transpose(1, 2))}
        for i in range(order + 1):
            arrays[f"q{i}"] = np32(caps[f"qn{i}"])
            arrays[f"dq{i}"] = np32(caps[f"qn{i}"].grad)
        for i in range(1, order):
            kv = caps[f"kv{i}"]
            v = kv.reshape(b, n, 2, 4, 16)[:, :, 1].transpose(1, 2)
            dv = kv.grad.reshape(b, n, 2, 4, 16)[:, :, 1].transpose(1, 2)
            arrays[f"v{i + 1}"] = np32(v)
            arrays[f"dv{i + 1}"] = np32(dv)
        save(f"chain_grad_o{order}", **arrays)


def vit_cases():
    # PolyViT forward (poly_attention/poly_vit.py:65-101), order 2 and 3
    for order in (2, 3):
        torch.manual_seed(60 + order)
        m = PolyViT(image_size=32, patch_size=8, num_classes=10, dim=64, depth=2, heads=4, mlp_dim=128,
                    dim_head=16, order=order, use_flash_kernel=False if order == 2 else None)
        img = torch.randn(2, 3, 32, 32)
        with torch.no_grad():
            y = m(img)
        save(f"vit_o{order}", img=np32(img), y=np32(y), **{f"p:{k}": v for k, v in state_np(m).items()})


def vit_full_case():
    # full-size PolyViT of BASELINE config 3 (poly_attention/poly_vit.py:65-101)
    # on 2 images: only the outputs are committed; weights and images are
    # rebuilt from seeds (tests/golden/seeded.py)
    from seeded import VIT_FULL, VIT_FULL_IMG_SEED, VIT_FULL_SEED, seeded_images, seeded_state_dict
    m = PolyViT(**VIT_FULL)
    sd = seeded_state_dict([(k, v.shape) for k, v in m.state_dict().items()], VIT_FULL_SEED)
    m.load_state_dict(sd)
    img = seeded_images(2, VIT_FULL_IMG_SEED)
    with torch.no_grad():
        y = m(img)
    save("vit_full", y=np32(y), img_checksum=np.float64(img.double().sum().item()),
         weight_checksum=np.float64(sum(v.double().abs().sum().item() for v in sd.values())))


CASES = {"ref_fn": ref_fn_cases, "mod2": mod2_cases, "modn": modn_cases, "vit": vit_cases, "vit_full": vit_full_case}

if __name__ == "__main__":
    torch.set_num_threads(4)
    for name in (sys.argv[1:] or list(CASES)):
        CASES[name]()
