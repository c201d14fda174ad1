from .layers import Embedding, Linear, RMSNorm, FeedForward, compute_ffn_hidden_dim
from .rope import RotaryEmbedding, precompute_rope
from .attention import GQAttention
from .decoder import Decoder

__all__ = [
    "Embedding", "Linear", "RMSNorm", "FeedForward", "compute_ffn_hidden_dim",
    "RotaryEmbedding", "precompute_rope", "GQAttention", "Decoder",
]
