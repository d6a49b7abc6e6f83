"""Attention backward (extension; the reference has none): dQ, dK, dV of the sm_100a
backward against the double-precision oracle (pinned to torch autograd in
test_oracle.py). Tolerance: the gradients pass through bf16 P and dS, as in
FlashAttention-2, so errors are bounded relative to each gradient's scale:
max |err| <= 2e-2 * max |ref| and mean |err| <= 1e-2 * mean |ref|."""
import numpy as np
import pytest
import torch

from oracle import oracle

pytestmark = pytest.mark.gpu


def _check(got, ref, name):
    g = got.float().cpu().numpy()
    err = np.abs(g - ref)
    scale_max, scale_mean = np.abs(ref).max(), np.abs(ref).mean()
    assert np.isfinite(g).all(), name
    assert err.max() <= 2e-2 * scale_max and err.mean() <= 1e-2 * scale_mean, (name, err.max(), scale_max,
                                                                                err.mean(), scale_mean)


@pytest.mark.parametrize("B,H,N,dist", [(1, 1, 128, "normal"), (1, 2, 256, "normal"), (2, 2, 300, "peaked"),
                                        (1, 1, 1, "normal"), (2, 3, 1024, "normal"), (1, 2, 777, "uniform")])
def test_backward_parity(B, H, N, dist):
    from blackflash_b200 import attention_backward, forward_lse
    from blackflash_b200.inputs import make_qkv
    q, k, v = make_qkv(B, H, N, dist=dist, seed=N + 11 * H, device="cuda")
    g = torch.Generator(device="cuda").manual_seed(N)
    do = torch.randn(q.shape, generator=g, device="cuda").to(torch.bfloat16)
    O, lse, _ = forward_lse(q, k, v, 0.125)
    dq, dk, dv = attention_backward(q, k, v, O, do, lse, 0.125)
    torch.cuda.synchronize()
    rq, rk, rv = oracle.attn_bwd(q.cpu(), k.cpu(), v.cpu(), do.cpu(), 0.125)
    _check(dv, rv, "dV")
    _check(dk, rk, "dK")
    _check(dq, rq, "dQ")


def test_autograd_function():
    from blackflash_b200 import blackflash_with_grad
    from blackflash_b200.inputs import make_qkv
    q, k, v = (t.requires_grad_(True) for t in make_qkv(1, 2, 256, seed=9, device="cuda"))
    o = blackflash_with_grad(q, k, v)
    do = torch.randn_like(o)
    o.backward(do)
    rq, rk, rv = oracle.attn_bwd(q.detach().cpu(), k.detach().cpu(), v.detach().cpu(), do.cpu(), 0.125)
    _check(q.grad, rq, "dQ")
    _check(k.grad, rk, "dK")
    _check(v.grad, rv, "dV")
