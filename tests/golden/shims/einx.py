"""Test-only stand-in for the ``einx`` package (absent from this image).

Only the three einx patterns that the reference's hot path uses are provided,
each implemented from the meaning of its pattern string:

- ``where('b j, b h i j, -> b h i j', m, s, v)``  key mask broadcast over h, i
  (poly_attention/poly_attention.py:76,102; n_poly_attention.py:254)
- ``where('b i, b h i j, -> b h i j', m, s, v)``  query mask broadcast over h, j
  (poly_attention/poly_attention.py:105; n_poly_attention.py:259)
- ``add('b h j, b h i j -> b h i j', l, s)``      per-key bias broadcast over i
  (poly_attention/poly_attention.py:109; n_poly_attention.py:288,307)

Any other pattern raises, so a silent mismatch is impossible.
"""
import torch


def where(pattern, cond, x, y):
    pattern = " ".join(pattern.split())
    if pattern == "b j, b h i j, -> b h i j":
        c = cond[:, None, None, :]
    elif pattern == "b i, b h i j, -> b h i j":
        c = cond[:, None, :, None]
    else:
        raise NotImplementedError(f"einx shim: unsupported where pattern {pattern!r}")
    return torch.where(c, x, torch.as_tensor(y, dtype=x.dtype, device=x.device))


def add(pattern, a, b):
    pattern = " ".join(pattern.split())
    if pattern == "b h j, b h i j -> b h i j":
        return a[..., None, :] + b
    raise NotImplementedError(f"einx shim: unsupported add pattern {pattern!r}")
