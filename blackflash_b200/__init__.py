"""BlackFlash-B200: a B200-native (sm_100a) attention forward behind BlackFlash's API.

    from blackflash_b200 import blackflash
    O = blackflash(Q, K, V)            # Q, K, V: [B, H, N, 64] bf16 CUDA

The compute path is libblackflash_b200.so (tcgen05 / TMA / TMEM kernel); there
is no CPU fallback.
"""
from .ops import (attention_backward, attention_partial, attention_partial_blocks, blackflash, blackflash_with_grad, blackflash_host, forward, forward_lse,  # noqa: F401
                  lse_merge_, to_bf16, wait_status)

__all__ = ["blackflash", "blackflash_with_grad", "attention_backward", "blackflash_host", "forward", "forward_lse", "attention_partial", "attention_partial_blocks", "lse_merge_", "to_bf16", "wait_status"]
