"""PolyViT, API- and state_dict-compatible with poly_attention/poly_vit.py:42-101.

Patch embedding, LayerNorms, MLPs and the head are PyTorch (cuBLAS); each
layer's attention core is the CUDA library (order 2 by default).
"""
from __future__ import annotations

import torch
from torch import nn
from torch.nn import Module, ModuleList

from .n_poly_attention import NPolyAttention
from .poly_attention import PolyAttention


def pair(t):
    return t if isinstance(t, tuple) else (t, t)


def posemb_sincos_2d(h, w, dim, temperature: int = 10000, dtype=torch.float32):
    """2-D sin-cos position table (poly_attention/poly_vit.py:19-30)."""
    assert dim % 4 == 0, "feature dimension must be multiple of 4 for sincos emb"
    omega = torch.arange(dim // 4) / (dim // 4 - 1)
    omega = 1.0 / (temperature ** omega)
    y, x = torch.meshgrid(torch.arange(h), torch.arange(w), indexing='ij')
    y = y.flatten()[:, None] * omega[None, :]
    x = x.flatten()[:, None] * omega[None, :]
    pe = torch.cat((x.sin(), x.cos(), y.sin(), y.cos()), dim=-1)
    return pe.type(dtype)


class _Patchify(Module):
    """'b c (h p1) (w p2) -> b (h w) (p1 p2 c)'."""

    def __init__(self, p1, p2):
        super().__init__()
        self.p1, self.p2 = p1, p2

    def forward(self, img):
        b, c, H, W = img.shape
        h, w = H // self.p1, W // self.p2
        t = img.view(b, c, h, self.p1, w, self.p2).permute(0, 2, 4, 3, 5, 1)
        return t.reshape(b, h * w, self.p1 * self.p2 * c)


def FeedForward(dim, hidden_dim):
    return nn.Sequential(nn.LayerNorm(dim), nn.Linear(dim, hidden_dim), nn.GELU(), nn.Linear(hidden_dim, dim))


class Transformer(Module):
    def __init__(self, dim, depth, heads, dim_head, mlp_dim, order=2, use_flash_kernel=None):
        super().__init__()
        self.norm = nn.LayerNorm(dim)
        self.layers = ModuleList([])
        for _ in range(depth):
            if order == 2:
                attn = PolyAttention(dim=dim, heads=heads, dim_head=dim_head, causal=False, prenorm=True,
                                     use_flash_kernel=use_flash_kernel)
            else:
                attn = NPolyAttention(dim=dim, order=order, heads=heads, dim_head=dim_head, causal=False, prenorm=True)
            self.layers.append(ModuleList([attn, FeedForward(dim, mlp_dim)]))

    def forward(self, x):
        for attn, ff in self.layers:
            x = attn(x) + x
            x = ff(x) + x
        return self.norm(x)


class PolyViT(Module):
    def __init__(self, *, image_size, patch_size, num_classes, dim, depth, heads, mlp_dim, channels=3, dim_head=64,
                 order=2, use_flash_kernel=None):
        super().__init__()
        ih, iw = pair(image_size)
        ph, pw = pair(patch_size)
        assert ih % ph == 0 and iw % pw == 0, 'Image dimensions must be divisible by the patch size.'
        patch_dim = channels * ph * pw
        self.to_patch_embedding = nn.Sequential(
            _Patchify(ph, pw), nn.LayerNorm(patch_dim), nn.Linear(patch_dim, dim), nn.LayerNorm(dim))
        self.pos_embedding = posemb_sincos_2d(h=ih // ph, w=iw // pw, dim=dim)
        self.transformer = Transformer(dim, depth, heads, dim_head, mlp_dim, order=order,
                                       use_flash_kernel=use_flash_kernel)
        self.linear_head = nn.Linear(dim, num_classes, bias=False)

    def forward(self, img):
        x = self.to_patch_embedding(img)
        x = x + self.pos_embedding.to(img.device, dtype=img.dtype)
        x = self.transformer(x)
        return self.linear_head(x.mean(dim=1))
