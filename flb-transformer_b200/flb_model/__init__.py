"""FLB-Transformer on this package's operators: the model (same math and parameter names as
the reference's models/FLB_Model.py) and a greedy decode loop for it."""
from .model import FLBAttentionLayer, FLBBlock, FLBTransformer, FLB_DEPENDENCIES
from .decode import greedy_decode

__all__ = ["FLBAttentionLayer", "FLBBlock", "FLBTransformer", "FLB_DEPENDENCIES",
           "greedy_decode"]
