"""Seeded weights and inputs for the full-size golden cases.

A full-size model's state_dict is far too large to commit as a fixture, so
the full-size cases commit only the reference's outputs and rebuild the
weights and inputs from a seed, with a procedure that depends on nothing but
the state_dict's names and shapes (not on either module's own init order):
every tensor, in sorted name order, is drawn from one CPU generator.
"""
import torch


def seeded_state_dict(names_shapes, seed):
    """names_shapes: iterable of (name, shape). Norm scales (names ending in
    'norm.weight' or 'norms.<i>.weight', or 1-D '.weight' of LayerNorm/RMSNorm)
    are 1 + 0.1 N(0,1); biases 0.02 N(0,1); matrices N(0,1) / sqrt(fan_in)."""
    g = torch.Generator().manual_seed(seed)
    out = {}
    for name, shape in sorted(names_shapes):
        shape = tuple(shape)
        x = torch.randn(shape, generator=g)
        if len(shape) == 1 and name.endswith("weight"):
            x = 1.0 + 0.1 * x
        elif len(shape) == 1:
            x = 0.02 * x
        else:
            fan_in = 1
            for s in shape[1:]:
                fan_in *= s
            x = x / fan_in ** 0.5
        out[name] = x
    return out


def seeded_images(batch, seed, size=256):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(batch, 3, size, size, generator=g)


VIT_FULL = dict(image_size=256, patch_size=32, num_classes=1000, dim=1024, depth=6, heads=16, dim_head=64,
                mlp_dim=2048, order=2)
VIT_FULL_SEED, VIT_FULL_IMG_SEED = 31, 32
