"""On-box comparison with the vendor library: torch SDPA's cuDNN backend on the same
inputs (non-causal and causal). Prints TFLOPS for both; asserts only that our
output matches cuDNN's within the parity tolerance (speed is reported, not asserted)."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _time(f, n=10):
    for _ in range(3):
        f()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(n):
        f()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / n


@pytest.mark.parametrize("causal", [False, True])
def test_versus_cudnn(causal):
    from torch.nn.attention import SDPBackend, sdpa_kernel
    from torch.nn.functional import scaled_dot_product_attention as sdpa

    from blackflash_b200 import blackflash
    from blackflash_b200.inputs import make_qkv
    B, H, N = 64, 64, 1024
    q, k, v = make_qkv(B, H, N, seed=1, device="cuda")
    fl = (2 if causal else 4) * B * H * N * N * 64
    try:
        with sdpa_kernel([SDPBackend.CUDNN_ATTENTION]):
            ref = sdpa(q, k, v, is_causal=causal, scale=0.125)
            ms_cudnn = _time(lambda: sdpa(q, k, v, is_causal=causal, scale=0.125))
    except RuntimeError as e:  # pragma: no cover - backend unavailable
        pytest.skip(f"cuDNN SDPA unavailable: {e}")
    out = blackflash(q, k, v, causal=causal)
    ms_ours = _time(lambda: blackflash(q, k, v, causal=causal))
    print(f"\n[{B},{H},{N}] causal={causal}: ours {fl / ms_ours / 1e9:.1f} TFLOPS, "
          f"cuDNN {fl / ms_cudnn / 1e9:.1f} TFLOPS")
    assert (out.float() - ref.float()).abs().max().item() <= 2e-2
