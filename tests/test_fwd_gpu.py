"""GPU parity of the sm_100a kernel against the CPU oracle (fp32 math attention).

Tolerance: on bf16 O, max |O - O_ref| <= 1e-2 and
mean |O - O_ref| <= 1e-3, O_ref the unrounded fp32 oracle on the same seeded inputs.
"""
import math

import numpy as np
import pytest
import torch

from golden_io import golden_cases, load_case
from oracle import oracle

pytestmark = pytest.mark.gpu

MAX_TOL = 1e-2
MEAN_TOL = 1e-3


def _dev():
    return torch.device("cuda:0")


def _errs(o_gpu: torch.Tensor, o_ref: np.ndarray):
    diff = np.abs(o_gpu.float().cpu().numpy() - o_ref)
    return float(diff.max()), float(diff.mean())


def _run_and_check(B, H, N, dist, seed, max_tol=MAX_TOL, mean_tol=MEAN_TOL, slices=None):
    from blackflash_b200 import forward_lse
    from blackflash_b200.inputs import make_qkv
    q, k, v = make_qkv(B, H, N, dist=dist, seed=seed, device=_dev())
    scale = 1.0 / math.sqrt(64)
    O, lse, mx = forward_lse(q, k, v, scale)
    torch.cuda.synchronize()
    qc, kc, vc = (t.reshape(B * H, N, 64) for t in (q, k, v))
    Oc, lsec, mxc = O.reshape(B * H, N, 64), lse.reshape(B * H, N), mx.reshape(B * H, N)
    idx = list(range(B * H)) if slices is None else slices
    idx_t = torch.tensor(idx, device=_dev())
    o_ref, lse_ref, mx_ref = oracle.attn_exact(qc[idx_t].cpu(), kc[idx_t].cpu(), vc[idx_t].cpu(), scale)
    mx_err, mean_err = _errs(Oc[idx_t], o_ref)
    assert mx_err <= max_tol and mean_err <= mean_tol, (B, H, N, dist, mx_err, mean_err)
    np.testing.assert_allclose(lsec[idx_t].cpu().numpy(), lse_ref, atol=2e-3, rtol=1e-4)
    np.testing.assert_allclose(mxc[idx_t].cpu().numpy(), mx_ref, atol=2e-3, rtol=1e-4)
    assert torch.isfinite(O).all()
    return mx_err, mean_err


def test_first_score_tile_debug_dump():
    """S = Q K^T of the first 128x128 tile straight from TMEM (checks TMA + UMMA descriptors)."""
    from blackflash_b200 import _lib
    from blackflash_b200.inputs import make_qkv
    q, k, v = make_qkv(1, 1, 256, dist="normal", seed=11, device=_dev())
    O = torch.empty_like(q)
    dbg = torch.full((128, 128), float("nan"), device=_dev())
    rc = _lib.load().blackflash_fwd_debug_s(q.data_ptr(), k.data_ptr(), v.data_ptr(), O.data_ptr(), dbg.data_ptr(),
                                            1, 1, 256, 64, 0.125, torch.cuda.current_stream().cuda_stream)
    _lib.check(rc, "debug_s")
    torch.cuda.synchronize()
    s_ref = (q[0, 0, :128].float() @ k[0, 0, :128].float().T).cpu().numpy()
    np.testing.assert_allclose(dbg.cpu().numpy(), s_ref, atol=1e-3, rtol=1e-3)


@pytest.mark.parametrize("case", golden_cases())
def test_reference_fixtures(case):
    """The reference's own gen_ref.py inputs: vs the oracle, and vs its bf16 SDPA o_ref."""
    from blackflash_b200 import blackflash
    c = load_case(case)
    m = c["meta"]
    to_t = lambda a: torch.from_numpy(a.astype(np.int16)).view(torch.bfloat16).to(_dev())
    q, k, v = to_t(c["q"]), to_t(c["k"]), to_t(c["v"])
    O = blackflash(q, k, v, m["scale"])
    torch.cuda.synchronize()
    o_exact, _, _ = oracle.attn_exact(c["q"], c["k"], c["v"], m["scale"])
    mx_err, mean_err = _errs(O, o_exact)
    assert mx_err <= MAX_TOL and mean_err <= MEAN_TOL
    # the reference harness's own check against o_ref.bin (src/main.cu:324, tol 0.02)
    o_ref = oracle.bf16_bits_to_f32(c["o_ref"])
    assert np.abs(O.float().cpu().numpy() - o_ref).max() < 0.02


@pytest.mark.parametrize("B,H,N,dist", [
    (2, 2, 512, "normal"),
    (4, 8, 1024, "normal"),
    (1, 1, 128, "normal"),
    (1, 1, 256, "uniform"),
    (3, 5, 384, "peaked"),      # odd B, H; 1.5 CTAs per slice
])
def test_parity_configs(B, H, N, dist):
    _run_and_check(B, H, N, dist, seed=B * 1000 + H * 10 + N)


@pytest.mark.parametrize("N", [1, 7, 64, 100, 129, 192, 255, 257, 1000])
def test_ragged_sequence_lengths(N):
    """N not a multiple of the 128-row tiles: masked KV tail, clipped stores."""
    _run_and_check(2, 3, N, "normal", seed=N)


def test_peaked_long_sequence_sampled():
    """BASELINE config 4 (8,16,8192), Q,K ~ N(0,3), V ~ U(-1,1); 4 slices checked against the oracle."""
    _run_and_check(8, 16, 8192, "peaked", seed=4, slices=[0, 37, 90, 127])


def test_large_config_sampled():
    """BASELINE config 3 (64,64,1024) at full size; a sample of slices checked against the oracle."""
    _run_and_check(64, 64, 1024, "normal", seed=3, slices=[0, 1, 777, 2048, 4095])


def test_deterministic_and_stream_ordered():
    from blackflash_b200 import blackflash
    from blackflash_b200.inputs import make_qkv
    q, k, v = make_qkv(2, 4, 640, seed=9, device=_dev())
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        O1 = blackflash(q, k, v)
        O2 = blackflash(q, k, v)
    s.synchronize()
    assert torch.equal(O1, O2)


def test_linearity_in_v_full_size():
    """Size-independent property: O(V1 + V2) = O(V1) + O(V2) within bf16 error."""
    from blackflash_b200 import blackflash
    from blackflash_b200.inputs import make_qkv
    q, k, v1 = make_qkv(16, 16, 1024, seed=21, device=_dev())
    _, _, v2 = make_qkv(16, 16, 1024, seed=22, device=_dev())
    v2 = v2 * 0.5
    # v1 + v2 exactly representable in bf16 is not guaranteed: compare against the sum of outputs in fp32.
    vs = (v1.float() + v2.float()).to(torch.bfloat16)
    O1, O2, Os = blackflash(q, k, v1), blackflash(q, k, v2), blackflash(q, k, vs)
    err = (Os.float() - (O1.float() + O2.float())).abs()
    assert err.max().item() < 2e-2 and err.mean().item() < 2e-3


def test_constant_v_rows_give_constant_output():
    """If every V row equals c, O = c regardless of scores (softmax weights sum to 1)."""
    from blackflash_b200 import blackflash
    from blackflash_b200.inputs import make_qkv
    q, k, _ = make_qkv(2, 2, 1536, dist="peaked", seed=5, device=_dev())
    c = torch.linspace(-1, 1, 64, device=_dev()).to(torch.bfloat16)
    v = c.view(1, 1, 1, 64).expand(2, 2, 1536, 64).contiguous()
    O = blackflash(q, k, v)
    assert (O.float() - c.float()).abs().max().item() <= 2 ** -8


def test_input_checks_raise():
    from blackflash_b200 import blackflash, forward
    q = torch.randn(1, 1, 64, 64, device=_dev(), dtype=torch.bfloat16)
    with pytest.raises(RuntimeError):
        forward(q.float(), q, q, 0.125)
    with pytest.raises(RuntimeError):
        forward(q.cpu(), q, q, 0.125)
    with pytest.raises(RuntimeError):
        forward(q.transpose(2, 3), q, q, 0.125)
    q96 = torch.randn(1, 1, 64, 96, device=_dev(), dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="d=64"):
        blackflash(q96, q96, q96)


def test_empty_input_returns_empty():
    from blackflash_b200 import blackflash
    q = torch.empty(0, 2, 64, 64, device=_dev(), dtype=torch.bfloat16)
    assert blackflash(q, q, q).shape == q.shape


def test_bounded_wait_timeout_reports_status():
    """A producer that never loads K: the consumers' bounded waits give up, the kernel
    returns, the status word names the wait site, and the context stays usable."""
    from blackflash_b200 import _lib, blackflash, wait_status
    from blackflash_b200.inputs import make_qkv
    wait_status(reset=True)
    q, k, v = make_qkv(1, 2, 512, seed=1, device=_dev())
    O = torch.empty_like(q)
    rc = _lib.load().blackflash_fwd_timeout_probe(q.data_ptr(), k.data_ptr(), v.data_ptr(), O.data_ptr(), 1, 2, 512,
                                                  64, 0.125, 20_000_000, torch.cuda.current_stream().cuda_stream)
    _lib.check(rc, "timeout probe")
    torch.cuda.synchronize()
    st = wait_status(reset=True)
    assert st != 0, "expected a wait-timeout status"
    assert wait_status(reset=False) == 0
    # context still healthy: a normal call works and is correct
    _run_and_check(1, 2, 512, "normal", seed=1)


@pytest.mark.parametrize("causal,chunks", [(False, 8), (True, 3), (False, 1)])
def test_host_buffer_api_matches_device_api(causal, chunks):
    """blackflash_host (pinned host tensors in and out, chunked and overlapped) equals the device API."""
    from blackflash_b200 import blackflash, blackflash_host
    from blackflash_b200.inputs import make_qkv
    q, k, v = make_qkv(3, 5, 700, seed=17)
    qh, kh, vh = (t.pin_memory() for t in (q, k, v))
    O_host = blackflash_host(qh, kh, vh, causal=causal, chunks=chunks)
    O_dev = blackflash(q.cuda(), k.cuda(), v.cuda(), causal=causal)
    torch.cuda.synchronize()
    assert not O_host.is_cuda
    assert torch.equal(O_host, O_dev.cpu())


def test_host_buffer_api_rejects_device_tensors():
    from blackflash_b200 import blackflash_host
    q = torch.zeros(1, 1, 64, 64, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(RuntimeError, match="host"):
        blackflash_host(q, q, q)
