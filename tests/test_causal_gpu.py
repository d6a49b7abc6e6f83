"""Causal mask (extension beyond the reference's non-causal kernel): parity against
the oracle's causal mode, same tolerance as the non-causal tests."""
import math

import numpy as np
import pytest
import torch

from oracle import oracle

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("B,H,N,dist", [(2, 3, 128, "normal"), (1, 2, 1024, "normal"), (2, 2, 777, "peaked"),
                                        (1, 1, 1, "normal"), (1, 4, 2560, "peaked"), (3, 1, 257, "uniform")])
def test_causal_parity(B, H, N, dist):
    from blackflash_b200 import forward_lse
    from blackflash_b200.inputs import make_qkv
    q, k, v = make_qkv(B, H, N, dist=dist, seed=N + H, device="cuda")
    O, lse, mx = forward_lse(q, k, v, 0.125, causal=True)
    torch.cuda.synchronize()
    o_ref, lse_ref, mx_ref = oracle.attn_exact(q.cpu(), k.cpu(), v.cpu(), 0.125, causal=True)
    d = np.abs(O.float().cpu().numpy() - o_ref)
    assert d.max() <= 1e-2 and d.mean() <= 1e-3, (d.max(), d.mean())
    np.testing.assert_allclose(lse.cpu().numpy(), lse_ref, atol=2e-3, rtol=1e-4)
    np.testing.assert_allclose(mx.cpu().numpy(), mx_ref, atol=2e-3, rtol=1e-4)


def test_causal_first_row_is_v0_and_noncausal_unchanged():
    from blackflash_b200 import blackflash
    from blackflash_b200.inputs import make_qkv
    q, k, v = make_qkv(2, 2, 640, seed=3, device="cuda")
    Oc = blackflash(q, k, v, causal=True)
    On = blackflash(q, k, v)
    torch.cuda.synchronize()
    # row 0 sees only key 0: its output is V[0] exactly (bf16 round trip)
    assert torch.equal(Oc[:, :, 0], v[:, :, 0])
    # the last row sees every key: causal and non-causal agree there
    assert (Oc[:, :, -1].float() - On[:, :, -1].float()).abs().max().item() <= 2 ** -8
