"""blackflash_bwd_noalloc, the backward for callers that cannot allocate device memory
(plugins whose host owns the whole device pool, or loops that cannot afford the
synchronisation of cudaMalloc / cudaFree). It uses a fixed scratch array inside the
library instead of a caller workspace.

Checked through the C ABI against blackflash_bwd (the entry point that takes a
workspace) on two calls in a row, which also covers the second call finding the
first call's data in the shared array, and once against the double-precision oracle. Tolerance as for the backward's parity
tests: max |err| <= 2e-2 * max |ref|, mean |err| <= 1e-2 * mean |ref|.
This file sorts last so that a run stopping at its first failure has run the rest."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _close(got, ref, name):
    g, r = got.float(), ref.float()
    err = (g - r).abs()
    assert torch.isfinite(g).all(), name
    assert err.max().item() <= 2e-2 * r.abs().max().item(), (name, err.max().item())
    assert err.mean().item() <= 1e-2 * r.abs().mean().item(), (name, err.mean().item())


def test_noalloc_backward_matches_workspace_backward():
    from blackflash_b200 import _lib, forward_lse
    from blackflash_b200.inputs import make_qkv
    lib = _lib.load()
    stream = torch.cuda.current_stream().cuda_stream
    for call, (B, H, N, seed) in enumerate([(2, 3, 300, 1), (1, 4, 1024, 2)]):
        q, k, v = make_qkv(B, H, N, dist="normal", seed=seed, device="cuda")
        do = torch.randn(q.shape, generator=torch.Generator(device="cuda").manual_seed(seed),
                         device="cuda").to(torch.bfloat16)
        O, lse, _ = forward_lse(q, k, v, 0.125)
        ins = [t.data_ptr() for t in (q, k, v, O, do, lse)]

        ref = [torch.empty_like(q) for _ in range(3)]
        nbytes = lib.blackflash_bwd_workspace_bytes(B, H, N, 64)
        ws = torch.empty(nbytes // 4, dtype=torch.float32, device="cuda")
        rc = lib.blackflash_bwd(*ins, *[t.data_ptr() for t in ref], ws.data_ptr(), nbytes, B, H, N, 64, 0.125, stream)
        _lib.check(rc, "blackflash_bwd")

        got = [torch.full_like(q, float("nan")) for _ in range(3)]
        rc = lib.blackflash_bwd_noalloc(*ins, *[t.data_ptr() for t in got], B, H, N, 64, 0.125, stream)
        _lib.check(rc, "blackflash_bwd_noalloc")
        torch.cuda.synchronize()
        for name, g, r in zip(("dQ", "dK", "dV"), got, ref):
            _close(g, r, f"call {call}: {name}")
        if call == 0:  # and, on its own, against the double-precision oracle
            from oracle import oracle
            exact = oracle.attn_bwd(q.cpu(), k.cpu(), v.cpu(), do.cpu(), 0.125)
            for name, g, r in zip(("dQ", "dK", "dV"), got, exact):
                _close(g, torch.from_numpy(r).cuda(), f"oracle: {name}")


def test_noalloc_backward_rejects_oversize():
    from blackflash_b200 import _lib
    lib = _lib.load()
    rc = lib.blackflash_bwd_noalloc(16, 16, 16, 16, 16, 16, 16, 16, 16, 64, 64, 1024, 64, 0.125, None)
    assert rc == _lib.BF_ERR_ARG and b"64 MiB" in lib.blackflash_last_error()
