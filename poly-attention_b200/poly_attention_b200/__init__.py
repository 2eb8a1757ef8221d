"""B200-native (sm_100a) poly attention: drop-in modules and functions for
lucidrains/poly-attention's hot path, backed by libpolyattn.so."""
from .core import (flash_poly_attention, poly_attention_chain, poly_attention_chain_cached,
                   poly_attention_order2, poly_attention_order2_cached)
from .host_stream import HostStreamedOrder2
from .n_poly_attention import NPolyAttention
from .ops import kernel_names, lse_merge, pass_bwd, pass_fwd
from .poly_attention import Order2PolyAttention, PolyAttention
from .poly_vit import PolyViT

__all__ = [
    "PolyAttention", "Order2PolyAttention", "NPolyAttention", "PolyViT", "flash_poly_attention",
    "poly_attention_order2", "poly_attention_order2_cached", "poly_attention_chain", "poly_attention_chain_cached",
    "pass_fwd", "pass_bwd", "lse_merge", "kernel_names", "HostStreamedOrder2",
]
