"""The reference's own kernel (kernel/flash_attn_mma.cu, compiled unchanged for
sm_100a into oracle/_ref/libref_kernel.so by oracle/Makefile) run on the same
inputs as ours: a checker for parity (both must agree with the oracle) and the
on-box comparator for speed. Skipped when oracle/_ref was not built (the
reference sources are only present in the build container).

The reference kernel assumes N % 64 == 0 (no KV tail masking), so only such
shapes are used."""
import ctypes
import math
import os

import numpy as np
import pytest
import torch

from oracle import oracle

pytestmark = pytest.mark.gpu
REF_LIB = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "oracle", "_ref",
                       "libref_kernel.so")
SYM = "_Z23flash_attn_naive_launchPK13__nv_bfloat16S1_S1_PS_PfS3_iiiifP11CUstream_st"


def _ref_launch():
    if not os.path.exists(REF_LIB):
        pytest.skip("oracle/_ref/libref_kernel.so not built")
    lib = ctypes.CDLL(REF_LIB)
    fn = getattr(lib, SYM)
    vp, i, f = ctypes.c_void_p, ctypes.c_int, ctypes.c_float
    fn.argtypes = [vp, vp, vp, vp, vp, vp, i, i, i, i, f, vp]
    fn.restype = None
    return fn


def _run_ref(fn, q, k, v, O, lm):
    B, H, N, d = q.shape
    fn(q.data_ptr(), k.data_ptr(), v.data_ptr(), O.data_ptr(), lm[0].data_ptr(), lm[1].data_ptr(), B, H, N, d,
       1.0 / math.sqrt(d), torch.cuda.current_stream().cuda_stream)


@pytest.mark.parametrize("B,H,N", [(2, 2, 512), (4, 8, 1024)])
def test_reference_and_ours_agree_with_oracle(B, H, N):
    from blackflash_b200 import blackflash
    from blackflash_b200.inputs import make_qkv
    fn = _ref_launch()
    q, k, v = make_qkv(B, H, N, seed=B + H + N, device="cuda")
    O_ref = torch.zeros_like(q)
    lm = (torch.empty(B, H, N, device="cuda"), torch.empty(B, H, N, device="cuda"))
    _run_ref(fn, q, k, v, O_ref, lm)
    O = blackflash(q, k, v)
    torch.cuda.synchronize()
    o_exact, _, _ = oracle.attn_exact(q.cpu(), k.cpu(), v.cpu(), 1.0 / math.sqrt(64))
    d_ref = np.abs(O_ref.float().cpu().numpy() - o_exact)
    d_ours = np.abs(O.float().cpu().numpy() - o_exact)
    print(f"\n[{B},{H},{N}] reference max/mean {d_ref.max():.2e}/{d_ref.mean():.2e}; "
          f"ours {d_ours.max():.2e}/{d_ours.mean():.2e}")
    assert d_ref.max() < 0.02  # the reference's own O tolerance (src/main.cu:324)
    assert d_ours.max() <= 1e-2 and d_ours.mean() <= 1e-3


def test_speed_versus_reference_kernel():
    """Same inputs, same device: TFLOPS of the reference kernel and of ours (printed)."""
    from blackflash_b200 import _lib
    from blackflash_b200.inputs import make_qkv
    fn = _ref_launch()
    lib = _lib.load()
    out = []
    for (B, H, N) in [(4, 8, 1024), (64, 64, 1024)]:
        q, k, v = make_qkv(B, H, N, seed=1, device="cuda")
        O = torch.empty_like(q)
        lm = (torch.empty(B, H, N, device="cuda"), torch.empty(B, H, N, device="cuda"))
        st = torch.cuda.current_stream().cuda_stream
        runs = {"reference": lambda: _run_ref(fn, q, k, v, O, lm),
                "ours": lambda: lib.blackflash_fwd(q.data_ptr(), k.data_ptr(), v.data_ptr(), O.data_ptr(), None, None,
                                                   B, H, N, 64, 0.125, st)}
        res = {}
        for name, f in runs.items():
            for _ in range(3):
                f()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(10):
                f()
            e1.record()
            torch.cuda.synchronize()
            res[name] = 4 * B * H * N * N * 64 / (e0.elapsed_time(e1) / 10 * 1e-3) / 1e12
        out.append((B, H, N, res))
        print(f"\n[{B},{H},{N}] reference kernel {res['reference']:.1f} TFLOPS, ours {res['ours']:.1f} TFLOPS "
              f"({res['ours'] / res['reference']:.1f}x)")
        assert res["ours"] > res["reference"]
        del q, k, v, O
