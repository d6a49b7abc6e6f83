"""The reference's Python entry point, `from blackflash import blackflash`
(reference blackflash/__init__.py:1-18): the same function name, arguments and
default scale 1/sqrt(d), served by the `blackflash_cuda` torch extension that this
repository builds at its root (csrc/torch_ext.cpp over libblackflash_b200.so)."""
import math

import blackflash_cuda


def blackflash(Q, K, V, scale=None):
    """O = softmax(scale * Q K^T) V for bf16 CUDA tensors [B, H, N, d] (d = 64, or 128
    as an extension); scale defaults to 1/sqrt(d)."""
    return blackflash_cuda.forward(Q, K, V, 1.0 / math.sqrt(Q.size(-1)) if scale is None else scale)


__all__ = ["blackflash"]
