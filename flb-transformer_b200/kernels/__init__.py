"""Additive-attention operator (B200 build of FLB-Transformer's kernels package)."""
from .additive_attention import FusedAdditiveAttentionFunc, fused_additive_attention

__all__ = ["FusedAdditiveAttentionFunc", "fused_additive_attention"]
