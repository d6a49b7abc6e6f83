"""The CPU oracle, pinned against the reference's own fixtures (tests/golden/,
made by the reference's profile/gen_ref.py) and cross-checked against a float64
numpy statement of the same formula."""
import numpy as np
import pytest

from golden_io import golden_cases, load_case
from oracle import oracle


@pytest.mark.parametrize("case", golden_cases())
def test_scores_match_gen_ref(case):
    c = load_case(case)
    m = c["meta"]
    for b in range(m["B"]):
        for h in range(m["H"]):
            s, p = oracle.scores(c["q"][b, h], c["k"][b, h], m["scale"])
            # gen_ref computes S in fp32 (matmul) - agreement to fp32 rounding of a 64-term dot product.
            np.testing.assert_allclose(s, c["s_ref"][b, h], rtol=0, atol=2e-6)
            np.testing.assert_allclose(p, c["p_ref"][b, h], rtol=0, atol=2e-7)


@pytest.mark.parametrize("case", golden_cases())
def test_exact_matches_gen_ref_output(case):
    c = load_case(case)
    m = c["meta"]
    o, lse, mx = oracle.attn_exact(c["q"], c["k"], c["v"], m["scale"])
    o_ref = oracle.bf16_bits_to_f32(c["o_ref"])
    # o_ref is torch SDPA rounded to bf16: |O| < 0.5, so one bf16 ulp is <= 2^-9.
    assert np.abs(o - o_ref).max() <= 2.0 ** -9
    # lse / rowmax against the fp32 S the reference saved.
    s = c["s_ref"].astype(np.float64)
    np.testing.assert_allclose(mx, s.max(-1), atol=1e-6)
    ref_lse = s.max(-1) + np.log(np.exp(s - s.max(-1, keepdims=True)).sum(-1))
    np.testing.assert_allclose(lse, ref_lse, atol=1e-5)


@pytest.mark.parametrize("case", golden_cases())
def test_fa2_restatement_within_reference_tolerance(case):
    """The reference kernel's algorithm lands within its own pinned O tolerance (src/main.cu:324)."""
    c = load_case(case)
    m = c["meta"]
    if m["N"] % 64:
        pytest.skip("the reference kernel assumes N % 64 == 0")
    o, lse, _ = oracle.attn_fa2(c["q"], c["k"], c["v"], m["scale"])
    o_ref = oracle.bf16_bits_to_f32(c["o_ref"])
    assert np.abs(o - o_ref).max() < 0.02


@pytest.mark.parametrize("shape,dist", [((1, 2, 37, 64), "normal"), ((2, 1, 130, 64), "peaked"),
                                        ((1, 1, 1, 64), "normal"), ((1, 3, 64, 64), "uniform")])
def test_exact_vs_numpy(shape, dist):
    from blackflash_b200.inputs import make_qkv
    q, k, v = make_qkv(*shape, dist=dist, seed=3)
    o, lse, _ = oracle.attn_exact(q, k, v, 0.125)
    o64, lse64 = oracle.attn_numpy(q, k, v, 0.125)
    np.testing.assert_allclose(o, o64, atol=1e-6, rtol=1e-6)
    np.testing.assert_allclose(lse, lse64, atol=1e-5)


def test_cross_attention_shapes():
    from blackflash_b200.inputs import make_qkv
    q, _, _ = make_qkv(1, 2, 40, seed=1)
    _, k, v = make_qkv(1, 2, 77, seed=2)
    o, lse, _ = oracle.attn_exact(q, k, v, 0.125)
    o64, lse64 = oracle.attn_numpy(q, k, v, 0.125)
    np.testing.assert_allclose(o, o64, atol=1e-6)
    np.testing.assert_allclose(lse, lse64, atol=1e-5)


def test_torch_math_matches_exact():
    from blackflash_b200.inputs import make_qkv
    q, k, v = make_qkv(2, 2, 96, seed=5)
    o = oracle.torch_math(q, k, v, 0.125).numpy()
    o2, _, _ = oracle.attn_exact(q, k, v, 0.125)
    np.testing.assert_allclose(o, o2, atol=2e-6)


@pytest.mark.parametrize("shape", [(1, 2, 37, 64), (2, 1, 300, 64), (1, 1, 1, 64)])
def test_causal_exact_vs_numpy(shape):
    from blackflash_b200.inputs import make_qkv
    q, k, v = make_qkv(*shape, dist="peaked", seed=11)
    o, lse, _ = oracle.attn_exact(q, k, v, 0.125, causal=True)
    o64, lse64 = oracle.attn_numpy(q, k, v, 0.125, causal=True)
    np.testing.assert_allclose(o, o64, atol=1e-6, rtol=1e-6)
    np.testing.assert_allclose(lse, lse64, atol=1e-5)


@pytest.mark.parametrize("B,H,N,d", [(1, 2, 64, 64), (2, 1, 100, 64), (1, 1, 37, 128)])
def test_backward_oracle_matches_torch_autograd(B, H, N, d):
    """The backward restatement against autograd of the fp32 math forward
    (reference tests/test_blackflash.py:16-19) on the same bf16 inputs."""
    import torch
    from blackflash_b200.inputs import make_qkv
    q, k, v = make_qkv(B, H, N, d=d, dist="normal", seed=N + d)
    g = torch.Generator().manual_seed(3)
    do = torch.randn(q.shape, generator=g).to(torch.bfloat16)
    scale = 1.0 / d ** 0.5
    qf, kf, vf = (t.double().requires_grad_(True) for t in (q, k, v))
    o = torch.softmax((qf @ kf.transpose(-1, -2)) * scale, dim=-1) @ vf
    o.backward(do.double())
    dq, dk, dv = oracle.attn_bwd(q, k, v, do, scale)
    for got, ref in ((dq, qf.grad), (dk, kf.grad), (dv, vf.grad)):
        np.testing.assert_allclose(got, ref.numpy(), rtol=1e-5, atol=1e-6)


def test_ref_data_writer_format(tmp_path):
    """tests/golden/make_ref_data.py writes gen_ref's layout (readable by golden_io) with
    the distribution keys, and its o_ref is the bf16 rounding of the torch fp32 formula."""
    import os
    import sys

    import torch
    from golden_io import GOLDEN_DIR, read_meta
    sys.path.insert(0, GOLDEN_DIR)
    from make_ref_data import write_ref_data
    out = str(tmp_path / "rd")
    write_ref_data(out, 1, 2, 96, dist="peaked", seed=3)
    m = read_meta(out)
    assert m["dist_q"] == "normal(0,3)" and m["dist_v"] == "uniform(-1,1)" and m["seed"] == 3
    shape = (m["B"], m["H"], m["N"], m["d"])
    assert shape == (1, 2, 96, 64) and abs(m["scale"] - 0.125) < 1e-9

    def bf16(fn):
        raw = np.fromfile(os.path.join(out, fn), dtype="<u2").reshape(shape)
        return torch.from_numpy(raw.astype(np.int16)).view(torch.bfloat16)
    q, k, v, o = (bf16(f) for f in ("q.bin", "k.bin", "v.bin", "o_ref.bin"))
    ref = oracle.torch_math(q, k, v, 0.125)
    assert (o.float() - ref).abs().max().item() <= 1e-2  # one bf16 rounding of |O| <= 1
    assert not os.path.exists(os.path.join(out, "s_ref.bin"))
