"""The reference's own Python import path against this repository:
`import blackflash_cuda` (the torch extension, reference binding/blackflash_ops.cu:57-59)
and `from blackflash import blackflash` (reference blackflash/__init__.py:1-18)."""
import math

import numpy as np
import pytest
import torch

from oracle import oracle


@pytest.fixture(scope="module")
def ext():
    from blackflash_b200.build import build_torch_ext
    build_torch_ext()
    import blackflash_cuda
    return blackflash_cuda


def test_extension_rejects_what_the_reference_rejects(ext):
    """Non-CUDA, non-bf16, non-contiguous inputs and d = 96 raise RuntimeError before any
    device work (reference binding/blackflash_ops.cu:24-34)."""
    x = torch.zeros(1, 1, 64, 64, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="CUDA bfloat16"):
        ext.forward(x, x, x, 0.125)
    with pytest.raises(RuntimeError, match="CUDA bfloat16"):
        ext.forward(x.float(), x.float(), x.float(), 0.125)
    from blackflash import blackflash
    with pytest.raises(RuntimeError):
        blackflash(x, x, x)


@pytest.mark.gpu
@pytest.mark.parametrize("B,H,N,d", [(2, 2, 512, 64), (1, 3, 200, 64), (1, 2, 256, 128)])
def test_reference_import_path_matches_oracle(ext, B, H, N, d):
    from blackflash import blackflash
    from blackflash_b200.inputs import make_qkv
    q, k, v = make_qkv(B, H, N, d=d, seed=B * 100 + N, device="cuda")
    o1 = blackflash(q, k, v)                                   # default scale 1/sqrt(d)
    o2 = ext.forward(q, k, v, 1.0 / math.sqrt(d))
    torch.cuda.synchronize()
    o_ref, _, _ = oracle.attn_exact(q.cpu(), k.cpu(), v.cpu(), 1.0 / math.sqrt(d))
    for o in (o1, o2):
        assert o.dtype == torch.bfloat16 and o.shape == q.shape
        err = np.abs(o.float().cpu().numpy() - o_ref)
        assert err.max() <= 1e-2 and err.mean() <= 1e-3
    assert torch.equal(o1, o2)


@pytest.mark.gpu
def test_extension_guards_and_shape_checks(ext):
    from blackflash_b200.inputs import make_qkv
    q, k, v = make_qkv(1, 1, 128, seed=3, device="cuda")
    with pytest.raises(RuntimeError, match="same shape"):
        ext.forward(q, k[:, :, :64].contiguous(), v, 0.125)
    with pytest.raises(RuntimeError, match="contiguous"):
        ext.forward(q.transpose(2, 3), k, v, 0.125)
    q96 = torch.zeros(1, 1, 64, 96, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(RuntimeError, match="d=64"):
        ext.forward(q96, q96, q96, 0.125)
    if torch.cuda.device_count() > 1:  # the guard launches on Q's device, not the current one
        q1, k1, v1 = (t.to("cuda:1") for t in (q, k, v))
        with torch.cuda.device(0):
            o = ext.forward(q1, k1, v1, 0.125)
        assert o.device == q1.device
        assert torch.equal(o.cpu(), ext.forward(q, k, v, 0.125).cpu())
