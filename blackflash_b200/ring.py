"""Sequence-parallel ("ring") attention forward over G ranks.

The reference has no multi-GPU mode. This mode serves BASELINE.json's
long-sequence configuration (B=1, H=32, N=65536, d=64 over 8 GPUs). Rank r holds
rows [r*N/G, (r+1)*N/G) of Q, K and V for every (b, h) slice. Over G steps each
rank attends its Q block to every KV block:

    step s: KV block of rank (r - s) mod G
            O_s, lse_s = partial attention (fp32 O normalised over the block)
            merge:  lse = log(e^lse_acc + e^lse_s)
                    O   = O_acc e^(lse_acc - lse) + O_s e^(lse_s - lse)
            meanwhile: send the current KV block to rank r+1 and receive the
            next one from rank r-1 (torch.distributed P2P; NCCL over NVLink on
            GPUs), so the transfer overlaps the step's kernel.

The received block lands in a local HBM buffer before any kernel reads it, so no
kernel reads peer memory and no TMA multicast is involved.

The schedule is independent of the compute: `partial_fn`, `merge_fn` and
`finalize_fn` default to the sm_100a kernels, and the CPU tests substitute
torch restatements to run the same schedule on gloo ranks.
"""
from __future__ import annotations

from typing import Callable

import torch
import torch.distributed as dist


def _default_partial(q, k, v, scale):
    from .ops import attention_partial
    return attention_partial(q, k, v, scale)


def _default_merge(o_acc, lse_acc, o_p, lse_p):
    from .ops import lse_merge_
    lse_merge_(o_acc, lse_acc, o_p, lse_p)


def _default_finalize(o_acc):
    from .ops import to_bf16
    return to_bf16(o_acc)


def ring_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float, group=None,
                   partial_fn: Callable = _default_partial, merge_fn: Callable = _default_merge,
                   finalize_fn: Callable = _default_finalize, return_lse: bool = False):
    """This rank's rows of softmax(scale Q K^T) V over the full (all-rank) sequence.

    q, k, v: [S, n_local, 64] bf16 (S = B*H slices), this rank's sequence block.
    Returns bf16 O [S, n_local, 64] (and the fp32 lse [S, n_local] if return_lse).
    """
    if dist.is_available() and dist.is_initialized():
        world, rank = dist.get_world_size(group), dist.get_rank(group)
    else:
        world, rank = 1, 0  # one process: the ring degenerates to a single partial step
    if k.shape != v.shape or q.shape[0] != k.shape[0]:
        raise RuntimeError("ring_attention: q [S,n,64] and k, v [S,m,64] with equal S required")
    nxt = dist.get_global_rank(group, (rank + 1) % world) if group is not None else (rank + 1) % world
    prv = dist.get_global_rank(group, (rank - 1) % world) if group is not None else (rank - 1) % world

    cur_k, cur_v = k, v
    n_spare = min(2, world - 1)
    spare = [(torch.empty_like(k), torch.empty_like(v)) for _ in range(n_spare)]
    o_acc = lse_acc = None
    for step in range(world):
        reqs = []
        if step < world - 1:
            rk, rv = spare[step % 2]
            ops = [dist.P2POp(dist.isend, cur_k, nxt, group), dist.P2POp(dist.isend, cur_v, nxt, group),
                   dist.P2POp(dist.irecv, rk, prv, group), dist.P2POp(dist.irecv, rv, prv, group)]
            reqs = dist.batch_isend_irecv(ops)
        o_p, lse_p = partial_fn(q, cur_k, cur_v, scale)
        if o_acc is None:
            o_acc, lse_acc = o_p, lse_p
        else:
            merge_fn(o_acc, lse_acc, o_p, lse_p)
        for r in reqs:
            r.wait()
        if step < world - 1:
            cur_k, cur_v = spare[step % 2]
    out = finalize_fn(o_acc)
    return (out, lse_acc) if return_lse else out
