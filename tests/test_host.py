"""Host-side logic on CPU: the C ABI library's exports, argument checking before
any device call, B x H sharding, and the ring schedule on gloo ranks."""
import math
import os
import re
import socket
import subprocess

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _header_functions():
    """Functions declared by the C ABI header and the diagnostic-hooks header."""
    text = "".join(open(os.path.join(REPO, "include", h)).read()
                   for h in ("blackflash_b200.h", "blackflash_b200_diag.h"))
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(blackflash_\w+)\s*\(", text)))


def test_library_exports_every_header_symbol():
    from blackflash_b200 import _lib
    from blackflash_b200.build import build_lib
    build_lib()
    lib = _lib.load()
    names = _header_functions()
    assert set(names) == set(_lib.EXPORTED)
    for n in names:
        assert hasattr(lib, n), n
    assert lib.blackflash_abi_version() == 1
    assert lib.blackflash_last_error() == b""


def test_reference_signature_symbol_exported():
    """flash_attn_naive_launch with the reference's exact C++ signature (include/flash_attn.cuh)."""
    from blackflash_b200.build import LIB_PATH, build_lib
    build_lib()
    out = subprocess.run(["nm", "-D", "--defined-only", LIB_PATH], capture_output=True, text=True).stdout
    sym = "_Z23flash_attn_naive_launchPK13__nv_bfloat16S1_S1_PS_PfS3_iiiifP11CUstream_st"
    assert sym in out


def test_argument_errors_without_device_work():
    """Invalid arguments are rejected by the library before any CUDA call."""
    from blackflash_b200 import _lib
    lib = _lib.load()
    rc = lib.blackflash_fwd(16, 16, 16, 16, None, None, 1, 1, 64, 96, 0.125, None)
    assert rc == _lib.BF_ERR_ARG and b"d=64" in lib.blackflash_last_error()
    rc = lib.blackflash_fwd(16, 16, 16, 16, None, None, 0, 1, 64, 64, 0.125, None)
    assert rc == _lib.BF_ERR_ARG
    rc = lib.blackflash_fwd(17, 16, 16, 16, None, None, 1, 1, 64, 64, 0.125, None)
    assert rc == _lib.BF_ERR_ARG and b"aligned" in lib.blackflash_last_error()
    rc = lib.blackflash_fwd(None, 16, 16, 16, None, None, 1, 1, 64, 64, 0.125, None)
    assert rc == _lib.BF_ERR_ARG
    rc = lib.blackflash_fwd_partial(16, 16, 16, None, None, 1, 64, 64, 64, 0.125, None)
    assert rc == _lib.BF_ERR_ARG
    for blocks, rows, skip in ((0, 128, -1), (2, 100, 0), (2, 128, 2), (1, 128, 0), (2, 128, -2)):
        rc = lib.blackflash_fwd_partial_blocks(16, 16, 16, 16, 16, 1, 64, blocks, rows, skip, 64, 0.125, None)
        assert rc == _lib.BF_ERR_ARG, (blocks, rows, skip)
    rc = lib.blackflash_lse_merge(16, 16, 16, 16, 4, 32, None)
    assert rc == _lib.BF_ERR_ARG
    assert lib.blackflash_lse_merge(16, 16, 16, 16, 0, 64, None) == _lib.BF_OK
    assert lib.blackflash_f32_to_bf16(16, 16, 0, None) == _lib.BF_OK


def test_backward_argument_errors_without_device_work():
    """The backward entry points reject bad arguments before any CUDA call."""
    from blackflash_b200 import _lib
    lib = _lib.load()
    assert lib.blackflash_bwd_workspace_bytes(1, 1, 128, 64) == 4 * (128 * 64 + 2 * 128)
    assert lib.blackflash_bwd_workspace_bytes(1, 1, 100, 64) == 4 * (100 * 64 + 2 * 128)  # vectors padded to 128
    assert lib.blackflash_bwd_workspace_bytes(1, 1, 128, 128) == 0  # d = 64 only
    ptrs = [16] * 10
    rc = lib.blackflash_bwd(*ptrs, 1 << 20, 1, 1, 128, 128, 0.125, None)
    assert rc == _lib.BF_ERR_ARG and b"d=64" in lib.blackflash_last_error()
    rc = lib.blackflash_bwd(*ptrs, 16, 1, 1, 128, 64, 0.125, None)
    assert rc == _lib.BF_ERR_ARG and b"workspace" in lib.blackflash_last_error()
    rc = lib.blackflash_bwd(*ptrs, 1 << 20, 0, 1, 128, 64, 0.125, None)
    assert rc == _lib.BF_ERR_ARG
    # no-workspace variant: problems beyond its fixed scratch are refused up front
    rc = lib.blackflash_bwd_noalloc(*ptrs[:9], 64, 64, 1024, 64, 0.125, None)
    assert rc == _lib.BF_ERR_ARG and b"64 MiB" in lib.blackflash_last_error()
    rc = lib.blackflash_bwd_noalloc(*ptrs[:9], 1, 1, 128, 128, 0.125, None)
    assert rc == _lib.BF_ERR_ARG and b"d=64" in lib.blackflash_last_error()


def test_python_checks_mirror_the_reference_binding():
    """Same failures as binding/blackflash_ops.cu:24-34: RuntimeError on CPU / non-bf16 / non-contiguous / d != 64."""
    from blackflash_b200 import blackflash, forward
    q = torch.zeros(1, 1, 64, 64, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="CUDA"):
        forward(q, q, q, 0.125)
    with pytest.raises(RuntimeError):
        blackflash(q.float(), q, q)


@pytest.mark.parametrize("total,world", [(4096, 1), (4096, 8), (4096, 3), (5, 8), (0, 2), (7, 7)])
def test_slice_range_partitions(total, world):
    from blackflash_b200.shard import slice_range
    spans = [slice_range(total, world, r) for r in range(world)]
    assert spans[0][0] == 0 and spans[-1][1] == total
    for (a0, a1), (b0, b1) in zip(spans, spans[1:]):
        assert a1 == b0
    sizes = [b - a for a, b in spans]
    assert max(sizes) - min(sizes) <= 1


def test_shard_bh_views():
    from blackflash_b200.shard import shard_bh
    t = torch.arange(2 * 3 * 4 * 2).reshape(2, 3, 4, 2)
    parts = [shard_bh(t, 4, r) for r in range(4)]
    assert torch.equal(torch.cat(parts).reshape(2, 3, 4, 2), t)


# ---------------------------------------------------------------- ring on gloo

def _cpu_partial(q, k, v, scale):
    s = torch.matmul(q.float(), k.float().transpose(-1, -2)) * scale
    lse = torch.logsumexp(s, dim=-1)
    o = torch.matmul(torch.softmax(s, dim=-1), v.float())
    return o.contiguous(), lse.contiguous()


def _cpu_merge(o_acc, lse_acc, o_p, lse_p):
    m = torch.maximum(lse_acc, lse_p)
    wa, wp = torch.exp(lse_acc - m), torch.exp(lse_p - m)
    tot = wa + wp
    o_acc.mul_((wa / tot)[..., None]).add_(o_p * (wp / tot)[..., None])
    lse_acc.copy_(m + torch.log(tot))


def _cpu_partial_blocks(q, kg, vg, scale, skip):
    """The gathered-block kernel's contract: keys are the used blocks, concatenated."""
    used = [g for g in range(kg.shape[0]) if g != skip]
    return _cpu_partial(q, torch.cat([kg[g] for g in used], dim=1), torch.cat([vg[g] for g in used], dim=1), scale)


def _ring_worker(rank, world, port, q, k, v, out_path, mode="ring"):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from blackflash_b200.ring import allgather_attention, ring_attention
    n = q.shape[1] // world
    sl = slice(rank * n, (rank + 1) * n)
    args = (q[:, sl].contiguous(), k[:, sl].contiguous(), v[:, sl].contiguous(), 0.125)
    if mode in ("ring", "ring2"):
        o, lse = ring_attention(*args, partial_fn=_cpu_partial, merge_fn=_cpu_merge, finalize_fn=lambda x: x,
                                return_lse=True, bidirectional=(mode == "ring2"), partial_blocks_fn=_cpu_partial_blocks)
    else:
        o, lse = allgather_attention(*args, partial_fn=_cpu_partial, partial_blocks_fn=_cpu_partial_blocks,
                                     merge_fn=_cpu_merge, finalize_fn=lambda x: x, return_lse=True)
    torch.save({"o": o, "lse": lse}, f"{out_path}.{rank}")
    dist.barrier()
    dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world", [2, 3])
def test_ring_schedule_on_gloo_matches_full_attention(world, tmp_path):
    from blackflash_b200.inputs import make_qkv
    from oracle import oracle
    q, k, v = make_qkv(1, 2, 96 * world, dist="peaked", seed=world)
    q, k, v = (t.reshape(2, 96 * world, 64) for t in (q, k, v))
    out = str(tmp_path / "ring")
    mp.spawn(_ring_worker, args=(world, _free_port(), q, k, v, out), nprocs=world, join=True)
    o = torch.cat([torch.load(f"{out}.{r}")["o"] for r in range(world)], dim=1).numpy()
    lse = torch.cat([torch.load(f"{out}.{r}")["lse"] for r in range(world)], dim=1).numpy()
    o_ref, lse_ref, _ = oracle.attn_exact(q, k, v, 0.125)
    np.testing.assert_allclose(o, o_ref, atol=2e-5)
    np.testing.assert_allclose(lse, lse_ref, atol=2e-4)


@pytest.mark.parametrize("world", [3, 4, 5])
def test_bidirectional_ring_on_gloo_matches_full_attention(world, tmp_path):
    """Both-way rotation: every foreign block arrives once, odd and even rank counts."""
    from blackflash_b200.inputs import make_qkv
    from oracle import oracle
    n = 128 * world
    q, k, v = make_qkv(1, 2, n, dist="peaked", seed=20 + world)
    q, k, v = (t.reshape(2, n, 64) for t in (q, k, v))
    out = str(tmp_path / "ring2")
    mp.spawn(_ring_worker, args=(world, _free_port(), q, k, v, out, "ring2"), nprocs=world, join=True)
    o = torch.cat([torch.load(f"{out}.{r}")["o"] for r in range(world)], dim=1).numpy()
    lse = torch.cat([torch.load(f"{out}.{r}")["lse"] for r in range(world)], dim=1).numpy()
    o_ref, lse_ref, _ = oracle.attn_exact(q, k, v, 0.125)
    np.testing.assert_allclose(o, o_ref, atol=2e-5)
    np.testing.assert_allclose(lse, lse_ref, atol=2e-4)


@pytest.mark.parametrize("world", [2, 3])
def test_allgather_schedule_on_gloo_matches_full_attention(world, tmp_path):
    from blackflash_b200.inputs import make_qkv
    from oracle import oracle
    n = 128 * world
    q, k, v = make_qkv(1, 2, n, dist="peaked", seed=10 + world)
    q, k, v = (t.reshape(2, n, 64) for t in (q, k, v))
    out = str(tmp_path / "ag")
    mp.spawn(_ring_worker, args=(world, _free_port(), q, k, v, out, "allgather"), nprocs=world, join=True)
    o = torch.cat([torch.load(f"{out}.{r}")["o"] for r in range(world)], dim=1).numpy()
    lse = torch.cat([torch.load(f"{out}.{r}")["lse"] for r in range(world)], dim=1).numpy()
    o_ref, lse_ref, _ = oracle.attn_exact(q, k, v, 0.125)
    np.testing.assert_allclose(o, o_ref, atol=2e-5)
    np.testing.assert_allclose(lse, lse_ref, atol=2e-4)


def test_build_tracks_every_source_and_header():
    """A file in csrc/ missing from the build's lists would leave a stale library after an
    edit (the rebuild check compares modification times of the listed files only)."""
    import glob

    from blackflash_b200 import build
    listed = set(build.SOURCES) | set(build.HEADERS) | {"harness.cu"}
    present = {os.path.basename(f) for f in glob.glob(os.path.join(build.CSRC, "*"))
               if f.endswith((".cu", ".cuh", ".h"))}
    assert present <= listed, sorted(present - listed)


def test_ring_entry_points_reject_bad_arguments_without_device_work():
    """blackflash_ring_* check their arguments before any CUDA call (csrc/ring_ipc.cu)."""
    import ctypes

    from blackflash_b200 import _lib
    lib = _lib.load()
    assert lib.blackflash_ring_handle_bytes() == 64
    ring = ctypes.c_void_p()
    handle = ctypes.create_string_buffer(64)
    for world, rank, bh, n, d in [(1, 0, 4, 128, 64), (4, 4, 4, 128, 64), (4, 0, 0, 128, 64), (4, 0, 4, 100, 64),
                                  (4, 0, 4, 128, 128)]:
        rc = lib.blackflash_ring_create(world, rank, bh, n, d, ctypes.byref(ring), handle)
        assert rc == _lib.BF_ERR_ARG, (world, rank, bh, n, d)
        assert lib.blackflash_last_error()
    assert lib.blackflash_ring_connect(None, handle) == _lib.BF_ERR_ARG
    assert lib.blackflash_ring_forward(None, 16, 16, 16, 16, None, 0.125, None) == _lib.BF_ERR_ARG
    assert lib.blackflash_ring_destroy(None) == _lib.BF_OK


def test_bidirectional_schedule_covers_every_block_once():
    from blackflash_b200.ring import bidirectional_schedule
    for world in range(1, 9):
        for rank in range(world):
            steps = bidirectional_schedule(world, rank)
            assert steps[0] == [rank]
            blocks = [b for st in steps for b in st]
            assert sorted(blocks) == list(range(world))
            assert len(steps) == world // 2 + 1
