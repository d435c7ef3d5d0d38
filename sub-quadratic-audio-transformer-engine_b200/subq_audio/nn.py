"""Neural-network module aliases (reference python/subq_audio/nn.py)."""
from .autograd import SubQAttentionFunction, SubQLinearAttention

SubQuadraticAttention = SubQLinearAttention

__all__ = ["SubQLinearAttention", "SubQuadraticAttention", "SubQAttentionFunction"]
