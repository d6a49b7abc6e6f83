// blackflash_cuda: the torch-extension module of the reference's Python path
// (binding/blackflash_ops.cu:18-59, built by setup.py:9-27 as `blackflash_cuda`),
// here a thin C++ shim over the C ABI of libblackflash_b200.so.
//
// forward(Q, K, V, scale) -> O keeps the reference's name, argument order and
// meaning, and raises RuntimeError (TORCH_CHECK) on the same bad inputs: non-CUDA
// or non-bf16 tensors, non-contiguous tensors, an unsupported head dimension.
// It differs from the reference in what a multi-GPU caller needs: a device guard
// on Q's device, K / V shape and device checks, no per-call l / m allocations,
// and a raised error (not exit()) when the launch fails. d = 128 is accepted as
// an extension of the reference's d = 64.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "../../include/blackflash_b200.h"

namespace {

torch::Tensor forward(const torch::Tensor& Q, const torch::Tensor& K, const torch::Tensor& V, double scale) {
    for (const torch::Tensor* t : {&Q, &K, &V}) {
        TORCH_CHECK(t->is_cuda() && t->scalar_type() == torch::kBFloat16, "Q, K and V must be CUDA bfloat16 tensors");
        TORCH_CHECK(t->is_contiguous(), "Q, K and V must be contiguous");
        TORCH_CHECK(t->dim() == 4, "Q, K and V must be [B, H, N, d]");
    }
    TORCH_CHECK(K.sizes() == Q.sizes() && V.sizes() == Q.sizes(), "Q, K and V must have the same shape");
    TORCH_CHECK(K.device() == Q.device() && V.device() == Q.device(), "Q, K and V must be on the same device");
    const int64_t B = Q.size(0), H = Q.size(1), N = Q.size(2), d = Q.size(3);
    TORCH_CHECK(d == 64 || d == 128, "BlackFlash supports d=64 and d=128");
    TORCH_CHECK(B <= INT32_MAX && H <= INT32_MAX && N <= INT32_MAX, "tensor dimensions exceed int range");

    const c10::cuda::CUDAGuard guard(Q.device());
    torch::Tensor O = torch::empty_like(Q);
    if (Q.numel() == 0) return O;
    const cudaStream_t stream = at::cuda::getCurrentCUDAStream(Q.device().index()).stream();
    const int rc = blackflash_fwd(Q.data_ptr(), K.data_ptr(), V.data_ptr(), O.data_ptr(), nullptr, nullptr, (int)B,
                                  (int)H, (int)N, (int)d, (float)scale, stream);
    TORCH_CHECK(rc == BF_OK, "blackflash_fwd failed (code ", rc, "): ", blackflash_last_error());
    return O;
}

}  // namespace

PYBIND11_MODULE(blackflash_cuda, m) {
    m.doc() = "BlackFlash-B200 attention forward (sm_100a) behind the reference's blackflash_cuda API";
    m.def("forward", &forward, "O = softmax(scale * Q K^T) V; bf16 [B, H, N, d], d = 64 or 128", pybind11::arg("Q"),
          pybind11::arg("K"), pybind11::arg("V"), pybind11::arg("scale"));
}
