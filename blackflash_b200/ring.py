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

By default the rotation runs both ways round the ring (`bidirectional=True`):
rank r receives blocks r-1, r-2, ... from the left and r+1, r+2, ... from the
right, two per step, and computes each pair in one gathered-block launch. The
classic one-way ring stays available (and is used for 2 ranks or per-rank blocks
that are not a multiple of 128 rows).

The received block lands in a local HBM buffer before any kernel reads it, so no
kernel reads peer memory and no TMA multicast is involved.

`allgather_attention` is the faster schedule for one NVSwitch node: an NCCL
all-gather of K and V into a local [G, S, n, 64] buffer runs while this rank's
own block is computed; then one kernel covers the other G-1 blocks straight
out of the gathered buffer (its producer maps KV tile -> block), and a single
LSE merge combines the two partials. Each KV block crosses NVLink once per rank
in one collective rather than G-1 dependent P2P steps, and G-2 merges go away.

The schedules are independent of the compute: `partial_fn`, `merge_fn` and
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
                   finalize_fn: Callable = _default_finalize, return_lse: bool = False,
                   bidirectional: bool = True, partial_blocks_fn: Callable | None = None):
    """This rank's rows of softmax(scale Q K^T) V over the full (all-rank) sequence.

    q, k, v: [S, n_local, 64] bf16 (S = B*H slices), this rank's sequence block.
    Returns bf16 O [S, n_local, 64] (and the fp32 lse [S, n_local] if return_lse).

    bidirectional=True (default) rotates KV both ways round the ring: at step s
    this rank holds the blocks of ranks r-s (arrived from the left) and r+s (from
    the right), computes both in one gathered-block launch, and forwards each one
    further in its direction. Two neighbours are in flight at once, and the
    G-1 foreign blocks arrive in floor(G/2) steps instead of G-1. NCCL's P2P
    bandwidth per peer pair falls as the rank count grows (measured on 8 B200s:
    81 GB/s per direction for one neighbour, 251 GB/s at 2 ranks), so a
    one-directional ring is transfer-bound there. bidirectional=False is the
    classic ring: one block per step, from the left.
    """
    if dist.is_available() and dist.is_initialized():
        world, rank = dist.get_world_size(group), dist.get_rank(group)
    else:
        world, rank = 1, 0  # one process: the ring degenerates to a single partial step
    if k.shape != v.shape or q.shape[0] != k.shape[0]:
        raise RuntimeError("ring_attention: q [S,n,64] and k, v [S,m,64] with equal S required")
    if world > 2 and bidirectional and k.shape[1] % 128 == 0:
        return _ring_bidirectional(q, k, v, scale, group, world, rank, partial_fn,
                                   partial_blocks_fn or _default_partial_blocks, merge_fn, finalize_fn, return_lse)
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


def bidirectional_schedule(world: int, rank: int) -> list[list[int]]:
    """The KV blocks (by owning rank) that `_ring_bidirectional` computes at each step
    on `rank`: [rank] first, then [r-s, r+s] for s = 1..nr and [r-s] for the one
    extra left step when G is even (nl = floor(G/2), nr = ceil(G/2) - 1)."""
    nl, nr = world // 2, (world + 1) // 2 - 1
    steps = [[rank]]
    for s in range(1, nl + 1):
        steps.append([(rank - s) % world] + ([(rank + s) % world] if s <= nr else []))
    return steps


def _ring_bidirectional(q, k, v, scale, group, world, rank, partial_fn, partial_blocks_fn, merge_fn, finalize_fn,
                        return_lse):
    """Both-way KV rotation (world >= 3). Blocks r-1 .. r-nl come from the left,
    r+1 .. r+nr from the right, nl = floor(G/2), nr = ceil(G/2) - 1, so every
    foreign block arrives exactly once. Step s >= 1 holds L_s (block r-s) in slot
    0 and R_s (block r+s, s <= nr) in slot 1 of a [2, S, n, 64] pair buffer."""
    g = (lambda x: dist.get_global_rank(group, x % world)) if group is not None else (lambda x: x % world)
    right, left = g(rank + 1), g(rank - 1)
    nl, nr = world // 2, (world + 1) // 2 - 1
    pair_k = [torch.empty((2,) + tuple(k.shape), dtype=k.dtype, device=k.device) for _ in range(2)]
    pair_v = [torch.empty_like(pair_k[0]) for _ in range(2)]

    def exchange(step, src_l, src_r):
        """Post the transfers that fill step+1's pair buffer."""
        dst_k, dst_v = pair_k[(step + 1) % 2], pair_v[(step + 1) % 2]
        ops = []
        if step + 1 <= nl:  # L_{s+1} = block r-s-1: the left neighbour forwards its L_s
            ops += [dist.P2POp(dist.isend, src_l[0], right, group), dist.P2POp(dist.isend, src_l[1], right, group),
                    dist.P2POp(dist.irecv, dst_k[0], left, group), dist.P2POp(dist.irecv, dst_v[0], left, group)]
        if step + 1 <= nr:  # R_{s+1} = block r+s+1: the right neighbour forwards its R_s
            ops += [dist.P2POp(dist.isend, src_r[0], left, group), dist.P2POp(dist.isend, src_r[1], left, group),
                    dist.P2POp(dist.irecv, dst_k[1], right, group), dist.P2POp(dist.irecv, dst_v[1], right, group)]
        return dist.batch_isend_irecv(ops) if ops else []

    reqs = exchange(0, (k, v), (k, v))
    o_acc, lse_acc = partial_fn(q, k, v, scale)
    for r in reqs:
        r.wait()
    for step in range(1, nl + 1):
        ck, cv = pair_k[step % 2], pair_v[step % 2]
        reqs = exchange(step, (ck[0], cv[0]), (ck[1], cv[1]))
        if step <= nr:
            o_p, lse_p = partial_blocks_fn(q, ck, cv, scale, -1)  # L_s and R_s in one launch
        else:
            o_p, lse_p = partial_fn(q, ck[0], cv[0], scale)
        merge_fn(o_acc, lse_acc, o_p, lse_p)
        for r in reqs:
            r.wait()
    out = finalize_fn(o_acc)
    return (out, lse_acc) if return_lse else out


def _default_partial_blocks(q, kg, vg, scale, skip):
    from .ops import attention_partial_blocks
    return attention_partial_blocks(q, kg, vg, scale, skip)


def allgather_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float, group=None,
                        partial_fn: Callable = _default_partial, partial_blocks_fn: Callable = _default_partial_blocks,
                        merge_fn: Callable = _default_merge, finalize_fn: Callable = _default_finalize,
                        return_lse: bool = False):
    """Same result as `ring_attention`, scheduled as all-gather + two partial kernels.

    q, k, v: [S, n, 64] bf16, this rank's sequence block; n a multiple of 128 when
    world > 1 (the gathered-block kernel's tiles never straddle two blocks).
    """
    if dist.is_available() and dist.is_initialized():
        world, rank = dist.get_world_size(group), dist.get_rank(group)
    else:
        world, rank = 1, 0
    if k.shape != v.shape or q.shape[0] != k.shape[0]:
        raise RuntimeError("allgather_attention: q [S,n,64] and k, v [S,m,64] with equal S required")
    if world == 1:
        o, lse = partial_fn(q, k, v, scale)
        out = finalize_fn(o)
        return (out, lse) if return_lse else out
    if k.shape[1] % 128:
        raise RuntimeError("allgather_attention: the per-rank KV block must have a multiple of 128 rows")
    kg = torch.empty((world,) + tuple(k.shape), dtype=k.dtype, device=k.device)
    vg = torch.empty_like(kg)
    if dist.get_backend(group) == "nccl":
        works = [dist.all_gather_into_tensor(kg, k.contiguous(), group=group, async_op=True),
                 dist.all_gather_into_tensor(vg, v.contiguous(), group=group, async_op=True)]
    else:
        works = [dist.all_gather(list(kg.unbind(0)), k.contiguous(), group=group, async_op=True),
                 dist.all_gather(list(vg.unbind(0)), v.contiguous(), group=group, async_op=True)]
    o_acc, lse_acc = partial_fn(q, k, v, scale)  # own block, overlapping the gather
    for w in works:
        w.wait()
    o_rem, lse_rem = partial_blocks_fn(q, kg, vg, scale, rank)
    merge_fn(o_acc, lse_acc, o_rem, lse_rem)
    out = finalize_fn(o_acc)
    return (out, lse_acc) if return_lse else out


class _IpcRing:
    """A blackflash_ring_* context (csrc/ring_ipc.cu) for one (group, shape, device)."""

    def __init__(self, group, world: int, rank: int, bh: int, n: int, device: torch.device):
        import ctypes

        from . import _lib
        self.lib = _lib.load()
        hb = self.lib.blackflash_ring_handle_bytes()
        handle = ctypes.create_string_buffer(hb)
        ptr = ctypes.c_void_p()
        with torch.cuda.device(device):
            _lib.check(self.lib.blackflash_ring_create(world, rank, bh, n, 64, ctypes.byref(ptr), handle),
                       "blackflash_ring_create")
        self.ptr = ptr
        handles = [None] * world
        dist.all_gather_object(handles, handle.raw, group=group)
        allh = ctypes.create_string_buffer(b"".join(handles), hb * world)
        with torch.cuda.device(device):
            _lib.check(self.lib.blackflash_ring_connect(self.ptr, allh), "blackflash_ring_connect")
        dist.barrier(group=group)  # every rank has opened its neighbours' buffers

    def __call__(self, q, k, v, scale, return_lse):
        from . import _lib
        out = torch.empty_like(q)
        lse = torch.empty(q.shape[:2], dtype=torch.float32, device=q.device) if return_lse else None
        with torch.cuda.device(q.device):
            rc = self.lib.blackflash_ring_forward(self.ptr, q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(),
                                                  lse.data_ptr() if lse is not None else None, float(scale),
                                                  torch.cuda.current_stream(q.device).cuda_stream)
        _lib.check(rc, "blackflash_ring_forward")
        return (out, lse) if return_lse else out

    def status(self) -> int:
        import ctypes
        v = ctypes.c_uint(0)
        self.lib.blackflash_ring_status(self.ptr, 1, ctypes.byref(v))
        return v.value

    def close(self):
        if self.ptr is not None:
            self.lib.blackflash_ring_destroy(self.ptr)
            self.ptr = None


_IPC_RINGS: dict = {}


def ipc_ring_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float, group=None,
                       return_lse: bool = False):
    """Same result as `ring_attention` (both-way schedule), with the KV rotation done by
    peer copies into the neighbours' memory over CUDA IPC (copy engines on NVLink) and
    GPU-side flags, all driven from C++ (blackflash_ring_forward). One process per GPU
    of one node; q, k, v: [S, n, 64] bf16 with n a multiple of 128. The ring context
    (buffers, IPC mappings) is created on first use for this group, shape and device
    and kept for later calls; `close_ipc_rings()` frees it."""
    world = dist.get_world_size(group) if dist.is_available() and dist.is_initialized() else 1
    if world == 1:
        return allgather_attention(q, k, v, scale, group=group, return_lse=return_lse)
    rank = dist.get_rank(group)
    if k.shape != v.shape or q.shape != k.shape or q.shape[-1] != 64:
        raise RuntimeError("ipc_ring_attention: q, k, v must all be [S, n, 64]")
    for t in (q, k, v):
        if not (t.is_cuda and t.dtype == torch.bfloat16 and t.is_contiguous()):
            raise RuntimeError("ipc_ring_attention: q, k, v must be contiguous CUDA bfloat16 tensors")
    key = (id(group), world, rank, q.shape[0], q.shape[1], q.device)
    ring = _IPC_RINGS.get(key)
    if ring is None:
        ring = _IPC_RINGS[key] = _IpcRing(group, world, rank, q.shape[0], q.shape[1], q.device)
    return ring(q, k, v, scale, return_lse)


def close_ipc_rings():
    """Free every ring context this process created (collective: call on all ranks)."""
    for r in _IPC_RINGS.values():
        r.close()
    _IPC_RINGS.clear()
