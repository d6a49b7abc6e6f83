"""Module-level stand-in for the reference's compiled extension `blackflash_cuda`
(binding/blackflash_ops.cu:57-59): exposes `forward(Q, K, V, scale)`."""
from .ops import forward  # noqa: F401
