"""Test-only stand-in for ``torch-einops-utils`` (absent from this image).

Provides the two helpers the reference's hot path calls, defined by their use
at the call sites (poly_attention/poly_attention.py:86-87,285-290,360-361;
n_poly_attention.py:206-213,281-302):

- ``safe_cat(ts, dim)``: concatenate the non-None entries; None if all are None.
- ``maybe(fn)``: a wrapper that passes None through and applies fn otherwise.
"""
import torch


def safe_cat(tensors, dim=0):
    tensors = [t for t in tensors if t is not None]
    if len(tensors) == 0:
        return None
    if len(tensors) == 1:
        return tensors[0]
    return torch.cat(tensors, dim=dim)


def maybe(fn):
    def inner(t, *args, **kwargs):
        if t is None:
            return None
        return fn(t, *args, **kwargs)
    return inner


def pack_with_inverse(*args, **kwargs):
    raise NotImplementedError("torch_einops_utils shim: pack_with_inverse is outside the hot path")
