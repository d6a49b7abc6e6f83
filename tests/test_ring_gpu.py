"""Sequence-parallel (ring) path on GPUs.

Single GPU: the ring's compute - partial attention per KV block, log-sum-exp
merge, bf16 cast - run over G blocks in one process must equal the full forward
and the oracle. Two or more GPUs: the real schedule over NCCL (one process per
GPU, P2P send/recv; both-way rotation from 3 ranks up), checked against the oracle."""
import math
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from oracle import oracle

pytestmark = pytest.mark.gpu


def test_partial_merge_equals_full_attention():
    from blackflash_b200 import attention_partial, forward_lse, lse_merge_, to_bf16
    from blackflash_b200.inputs import make_qkv
    S, N, G = 6, 1536, 4
    q, k, v = make_qkv(1, S, N, dist="peaked", seed=31, device="cuda")
    q3, k3, v3 = (t.reshape(S, N, 64) for t in (q, k, v))
    blk = N // G
    o_acc = lse_acc = None
    for b in range(G):
        o_p, l_p = attention_partial(q3, k3[:, b * blk:(b + 1) * blk].contiguous(),
                                     v3[:, b * blk:(b + 1) * blk].contiguous(), 0.125)
        if o_acc is None:
            o_acc, lse_acc = o_p, l_p
        else:
            lse_merge_(o_acc, lse_acc, o_p, l_p)
    o_ring = to_bf16(o_acc)
    O, lse, _ = forward_lse(q, k, v, 0.125)
    torch.cuda.synchronize()
    o_ref, lse_ref, _ = oracle.attn_exact(q3.cpu(), k3.cpu(), v3.cpu(), 0.125)
    d = np.abs(o_ring.float().cpu().numpy() - o_ref)
    assert d.max() <= 1e-2 and d.mean() <= 1e-3
    np.testing.assert_allclose(lse_acc.cpu().numpy(), lse_ref, atol=2e-3)
    assert (o_ring.float() - O.reshape(S, N, 64).float()).abs().max().item() <= 1e-2


def test_partial_ragged_blocks():
    """Partial attention with Nq != Nkv and ragged sizes (the masked KV tail)."""
    from blackflash_b200 import attention_partial
    from blackflash_b200.inputs import make_qkv
    q, _, _ = make_qkv(1, 3, 300, seed=1, device="cuda")
    _, k, v = make_qkv(1, 3, 457, seed=2, device="cuda")
    q3, k3, v3 = q.reshape(3, 300, 64), k.reshape(3, 457, 64), v.reshape(3, 457, 64)
    o, lse = attention_partial(q3, k3, v3, 0.125)
    torch.cuda.synchronize()
    o_ref, lse_ref, _ = oracle.attn_exact(q3.cpu(), k3.cpu(), v3.cpu(), 0.125)
    assert np.abs(o.cpu().numpy() - o_ref).max() <= 1e-2
    np.testing.assert_allclose(lse.cpu().numpy(), lse_ref, atol=2e-3)


@pytest.mark.parametrize("skip", [-1, 0, 2, 3])
def test_partial_blocks_matches_oracle(skip):
    """Gathered-block kernel: keys are blocks [G, S, n, 64] minus `skip`, concatenated."""
    from blackflash_b200 import attention_partial_blocks
    from blackflash_b200.inputs import make_qkv
    S, nq, n, G = 3, 300, 256, 4
    q, _, _ = make_qkv(1, S, nq, seed=41, device="cuda")
    _, kg, vg = make_qkv(G, S, n, dist="peaked", seed=42, device="cuda")  # [G, S, n, 64]
    q3 = q.reshape(S, nq, 64)
    o, lse = attention_partial_blocks(q3, kg, vg, 0.125, skip)
    torch.cuda.synchronize()
    used = [g for g in range(G) if g != skip]
    k_cat = torch.cat([kg[g] for g in used], dim=1).cpu()
    v_cat = torch.cat([vg[g] for g in used], dim=1).cpu()
    o_ref, lse_ref, _ = oracle.attn_exact(q3.cpu(), k_cat, v_cat, 0.125)
    d = np.abs(o.cpu().numpy() - o_ref)
    assert d.max() <= 1e-2 and d.mean() <= 1e-3
    np.testing.assert_allclose(lse.cpu().numpy(), lse_ref, atol=2e-3)


def test_partial_blocks_rejects_unaligned_blocks():
    from blackflash_b200 import attention_partial_blocks
    q = torch.zeros(2, 128, 64, device="cuda", dtype=torch.bfloat16)
    kg = torch.zeros(2, 2, 192, 64, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="multiple of 128"):
        attention_partial_blocks(q, kg, kg, 0.125, 0)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _ring_worker(rank, world, port, qkv, out, mode="ring"):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    from blackflash_b200.ring import allgather_attention, close_ipc_rings, ipc_ring_attention, ring_attention
    q, k, v = (t.cuda() for t in qkv)
    n = q.shape[1] // world
    sl = slice(rank * n, (rank + 1) * n)
    args = (q[:, sl].contiguous(), k[:, sl].contiguous(), v[:, sl].contiguous(), 0.125)
    if mode == "allgather":
        o = allgather_attention(*args)
    elif mode == "ipc":
        # Two calls on the same ring context: the second must not see the first call's
        # blocks. O is linear in V, so the first call (V negated) must give -O up to bf16
        # rounding (the tensor core's accumulation is not exactly sign-symmetric); a stale
        # block would differ by O(1).
        o2 = ipc_ring_attention(args[0], args[1], (-args[2]).contiguous(), 0.125)
        o = ipc_ring_attention(*args)
        torch.cuda.synchronize()
        assert (o2.float() + o.float()).abs().max().item() <= 1e-2, "second call on the ring saw stale data"
        close_ipc_rings()
    else:
        o = ring_attention(*args, bidirectional=(mode == "ring"))
    torch.save(o.cpu(), f"{out}.{rank}")
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs >= 2 GPUs")
@pytest.mark.parametrize("mode", ["ring", "ring1", "allgather", "ipc"])
def test_ring_over_nccl(tmp_path, mode):
    from blackflash_b200.inputs import make_qkv
    world = min(torch.cuda.device_count(), 8)  # at 8 ranks the both-way ring runs nl=4, nr=3
    S, N = 4, 512 * world
    q, k, v = (t.reshape(S, N, 64) for t in make_qkv(1, S, N, seed=77))
    out = str(tmp_path / "ring")
    mp.spawn(_ring_worker, args=(world, _free_port(), (q, k, v), out, mode), nprocs=world, join=True)
    o = torch.cat([torch.load(f"{out}.{r}") for r in range(world)], dim=1).float().numpy()
    o_ref, _, _ = oracle.attn_exact(q, k, v, 0.125)
    d = np.abs(o - o_ref)
    assert d.max() <= 1e-2 and d.mean() <= 1e-3


def test_config5_per_rank_schedules_on_one_gpu():
    """BASELINE config 5 (B=1 H=32 N=65536, N(0,1)) at its own shape: every per-rank
    computation of the 8-rank both-way ring (own block, then the pairs L_s / R_s in one
    gathered-block launch each, merged step by step in `bidirectional_schedule` order)
    and of the all-gather schedule (own block + one launch over the other 7 blocks),
    run in one process on one GPU. Sampled query rows of three heads on three ranks
    are checked against the oracle over all 65536 keys; every rank's two schedules must
    agree with each other."""
    from blackflash_b200 import attention_partial, attention_partial_blocks, lse_merge_, to_bf16
    from blackflash_b200.inputs import make_qkv
    from blackflash_b200.ring import bidirectional_schedule
    H, N, G = 32, 65536, 8
    n = N // G
    q, k, v = (t.reshape(H, N, 64) for t in make_qkv(1, H, N, seed=5005, device="cuda"))
    kb = torch.stack([k[:, r * n:(r + 1) * n] for r in range(G)])  # [G, H, n, 64], as all-gathered
    vb = torch.stack([v[:, r * n:(r + 1) * n] for r in range(G)])
    heads, rows = [0, 13, 31], torch.arange(0, n, 32)[:256]
    for r in range(G):
        qr = q[:, r * n:(r + 1) * n].contiguous()
        steps = bidirectional_schedule(G, r)
        assert sorted(b for st in steps for b in st) == list(range(G))
        o_acc, lse_acc = attention_partial(qr, kb[r], vb[r], 0.125)
        for st in steps[1:]:
            if len(st) == 2:
                o_p, l_p = attention_partial_blocks(qr, kb[st].contiguous(), vb[st].contiguous(), 0.125, -1)
            else:
                o_p, l_p = attention_partial(qr, kb[st[0]], vb[st[0]], 0.125)
            lse_merge_(o_acc, lse_acc, o_p, l_p)
        o_ring = to_bf16(o_acc)
        o_ag, lse_ag = attention_partial(qr, kb[r], vb[r], 0.125)
        o_rem, l_rem = attention_partial_blocks(qr, kb, vb, 0.125, r)
        lse_merge_(o_ag, lse_ag, o_rem, l_rem)
        o_ag = to_bf16(o_ag)
        torch.cuda.synchronize()
        assert (o_ring.float() - o_ag.float()).abs().max().item() <= 4e-3
        assert (lse_acc - lse_ag).abs().max().item() <= 1e-3
        if r not in (0, 3, 7):
            continue
        for h in heads:
            o_ref, lse_ref, _ = oracle.attn_exact(qr[h, rows].cpu(), k[h].cpu(), v[h].cpu(), 0.125)
            for o in (o_ring, o_ag):
                d = np.abs(o[h, rows].float().cpu().numpy() - o_ref)
                assert d.max() <= 1e-2 and d.mean() <= 1e-3, (r, h, d.max(), d.mean())
            np.testing.assert_allclose(lse_acc[h, rows].cpu().numpy(), lse_ref, atol=2e-3)
